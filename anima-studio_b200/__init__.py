"""anima-studio B200: the Anima DiT denoising hot path on sm_100a.

The package directory name carries a hyphen, so import it with
``importlib.import_module("anima-studio_b200")`` (see ``load_package`` in the repository's
entry points). Submodules:

  device    CUDA context, tensors and the C-ABI binding (libanima_b200.so)
  ops       the operator surface of the reference's app/gpu/ops.js
  weights   comfy_quant linear layouts (app/weights.js)
  lora      LoRA side paths (app/lora.js)
  dit       AnimaDiT: timeCond, prepareContext, forward (app/models/dit.js)
  pipeline  Euler / CFG sampling over the DiT (app/pipeline.js, app/samplers.js)
  quant     offline ConvRot quantizers (tools/quant.py)
  synthetic seeded synthetic checkpoints in the comfy_quant layout
"""

__all__ = ["device", "ops", "weights", "lora", "dit", "pipeline", "quant", "synthetic"]
