/*
 * anima_b200.h — C ABI of the B200 (sm_100a) backend for the Anima DiT denoising path.
 *
 * It replaces the WebGPU operator surface of the reference (app/gpu/ops.js + app/gpu/device.js)
 * for the DiT forward (app/models/dit.js:196-325). Each entry point below names the reference
 * interface it stands in for. Conventions:
 *   - Every call returns an anima_status; 0 is success. anima_last_error() gives the message of
 *     the calling thread's last failure. No exceptions cross the ABI.
 *   - All pointers are device pointers unless stated; sizes and strides are in elements.
 *   - Calls are asynchronous on the context's stream (like the reference's recorded dispatches,
 *     app/gpu/device.js:170-216); device-side faults and timeouts surface at anima_sync(), as the
 *     reference surfaces WebGPU validation errors at read/sync (device.js:224-231).
 *   - A context is owned by one host thread at a time (the reference's single worker thread).
 *   - Every call runs on its context's device, whatever device the calling thread has current, and
 *     leaves the thread's current device as it found it; one thread may drive contexts on several
 *     GPUs in turn. The context's stream must belong to its device.
 */
#ifndef ANIMA_B200_H
#define ANIMA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct anima_ctx anima_ctx;

typedef enum {
  ANIMA_OK = 0,
  ANIMA_ERR_ARG = 1,          /* bad shape, stride, alignment or enum value */
  ANIMA_ERR_CUDA = 2,         /* a CUDA runtime/driver call failed */
  ANIMA_ERR_DEVICE = 3,       /* a kernel reported a fault or a timed-out wait */
  ANIMA_ERR_UNSUPPORTED = 4,  /* valid request this build does not implement */
} anima_status;

typedef enum { ANIMA_F32 = 0, ANIMA_BF16 = 1, ANIMA_F16 = 2, ANIMA_I8 = 3, ANIMA_U8 = 4 } anima_dtype;
typedef enum { ANIMA_ACT_NONE = 0, ANIMA_ACT_GELU = 1, ANIMA_ACT_SILU = 2 } anima_act;

/* Weight kinds of app/weights.js:118-146 ({kind: "i8" | "w4" | "bf16"}) plus fp32 (LoRA A/B). */
typedef enum { ANIMA_W_I8 = 0, ANIMA_W_W4 = 1, ANIMA_W_BF16 = 2, ANIMA_W_F32 = 3, ANIMA_W_F16 = 4 } anima_weight_kind;

/* Rotated, per-token quantized activation rows (the "xr" input of ops.linear, ops.js:48-54):
 *   x[m, k] ~= scale[m] * (hi[m, k] + lo[m, k] / 254)
 * lo == NULL is the one-plane W8A8 form (x ~= scale * hi). hi/lo are row-major int8 [rows, ld]. */
typedef struct {
  int rows, cols, ld;
  int8_t* hi;
  int8_t* lo;
  float* scale;
} anima_qact;

/* A linear layer's weights in the comfy_quant layout (app/weights.js:118-146).
 *   I8  : data = int8 codes [N, K], scale = weight_scale [N]
 *   W4  : data = packed nibbles [N, K/2] (low nibble = even k), s_rel = fp8-e4m3 [N, K/16],
 *         codebook = [16], scale = weight_s_channel [N]
 *   BF16: data = bf16 [N, K];  F32: data = fp32 [N, K];  F16: data = fp16 [N, K] (anima_matmul
 *         only: the LoRA up-projection)
 * ConvRot layers (I8, W4) take rotated inputs, as in the reference (ops.js:35). */
typedef struct {
  int kind, N, K;
  const void* data;
  const float* scale;
  const uint8_t* s_rel;
  const float* codebook;
  const float* bias;
} anima_weight;

typedef enum {
  ANIMA_OUT_STORE = 0,          /* out[m, n] = y                                               */
  ANIMA_OUT_RESID = 1,          /* out[m, n] += (gate ? gate[gate_off + n] : 1) * y, fp32 out  */
  ANIMA_OUT_QKV_NORM_ROPE = 2,  /* per-head RMSNorm + split-half RoPE on q/k columns           */
  ANIMA_OUT_HEAD_NORM = 3,      /* per-head RMSNorm with norm_q on every head, no RoPE         */
} anima_out_mode;

/* Epilogue of anima_linear, in the reference's order (app/gpu/gemm.js:186-192):
 * y = acc * a_scale[m] * w_scale[n] (+ bias[n]) (+ add[m, n]) -> act -> output mode. */
typedef struct {
  int act;
  const float* add;
  int ld_add;
  int out_mode;
  int out_dtype;
  void* out;
  int ldo;
  const float* gate;
  int gate_off;
  const float* norm_q; /* [128] */
  const float* norm_k; /* [128] */
  const float* rope;   /* cos [rope_rows, 64] followed by sin [rope_rows, 64]; row = m % rope_rows */
  int rope_rows;
  int n_q;             /* QKV: columns [0, n_q) q heads, [n_q, 2 n_q) k heads, the rest v */
  float eps;
  /* LoRA side paths added in the epilogue before the activation (ops.js:55-57, 70-87):
     y[m, n] += sum_{i < r_e} t[m, r0_e + i] * lora_bt[r0_e + i, n] for the entry e whose
     columns [off_e, off_e + n_e) hold n, where t[m, j] = lora_t[m, j] (+ lora_t[m, lora_t_lo + j]
     when lora_t_lo > 0: x_r A^T computed as two partial products, e.g. by anima_linear with A in two
     int8 planes). lora_t [M, ld_t] holds x_r A^T of all entries stacked (or anima_lora_down's
     result); lora_bt [R, ld_bt] holds scale_e * B_e^T in the entry's columns (only those are read).
     Entries: off and n multiples of 128, r a multiple of 4 and at most 32, at most 4 entries;
     lora_t NULL = none. The epilogue multiplies fp16 copies of t and lora_bt with fp32 sums
     (the delta is a small part of y; it adds ~2^-11 of the delta). */
  const float* lora_t;
  int ld_t;
  int lora_t_lo;
  const float* lora_bt;
  int ld_bt;
  int lora_count;
  int lora_off[4], lora_n[4], lora_r0[4], lora_r[4];
  /* Sequence-parallel k|v exchange (QKV_NORM_ROPE only; no reference counterpart): when
     peer_count > 0 the k and v columns [n_q, N) do not go to out; every 32-row piece of them is
     stored instead into peer_kv[0..peer_count), each rank's gathered k|v buffer
     [items, peer_item_rows, N - n_q] (dtype out_dtype, 16-byte aligned) as mapped in this process
     (anima_ipc_open; this rank's own buffer included), at row peer_row0 + m % peer_rows of item
     m / peer_rows. peer_rows is a multiple of 32 dividing M; follow with anima_peer_barrier before
     any rank reads its buffer. Only TMA stores touch peer memory. */
  int peer_count;
  void* peer_kv[8];
  int peer_row0, peer_rows, peer_item_rows;
} anima_linear_opts;

typedef struct {
  int batch, heads, head_dim, Lq, Lk;
  int dtype;               /* ANIMA_BF16 or ANIMA_F16 for q/k/v (ANIMA_F32 too when group > 1,
                              causal or head_dim 64: the text models' path) */
  const void* q; long long ldq, q_bstride; int q_off;
  const void* k; long long ldk, k_bstride; int k_off;
  const void* v; long long ldv, v_bstride; int v_off;
  void* out; long long ldo, o_bstride; int out_dtype; /* F32, BF16 or F16 */
  const int* key_len;      /* [batch] keys >= key_len[b] are masked; NULL = all Lk keys.
                              k_bstride == v_bstride == 0 with batch > 1 shares one K/V and key_len[0]. */
  float scale;             /* softmax scale, 1/sqrt(head_dim) in the reference */
  int group;               /* q heads per k/v head (GQA, ops.js:166 `group`); 0 or 1 = none */
  int causal;              /* key j visible to query i only when j <= i (ops.js:166 `causal`) */
} anima_attention_args;

/* ---------------------------------------------------------------- runtime (device.js GPU) */
/* GPU.create (device.js:61-87). */
int anima_ctx_create(int device, anima_ctx** out);
int anima_ctx_destroy(anima_ctx* ctx);
/* Run subsequent calls on this CUDA stream (cudaStream_t; NULL = legacy default stream). */
int anima_ctx_set_stream(anima_ctx* ctx, void* stream);
/* How anima_attention spreads work over the SMs (no reference counterpart: the reference's WGSL
 * dispatch has no such choice). -1 (default, or the ANIMA_ATTN_STREAMK environment variable at
 * context creation): stream-K split of the key blocks when the last wave of whole units would leave
 * more than 5% of the SMs idle; 0: whole units only; 1: stream-K wherever legal (no key_len, at
 * least one unit per SM). Results of the two schedules differ by fp32 rounding only. */
int anima_ctx_set_attention_split(anima_ctx* ctx, int mode);
/* gpu.sync (device.js:218-232): wait for the stream, then report device-side errors. */
int anima_sync(anima_ctx* ctx);
const char* anima_last_error(void);
/* gpu.empty / Tensor.release (device.js:20-23,124-128), plain device allocations. */
int anima_alloc(anima_ctx* ctx, size_t bytes, void** out);
int anima_free(anima_ctx* ctx, void* ptr);
/* gpu.fromArray/upload and gpu.read (device.js:130-156,218-224): host <-> device copies. */
int anima_upload(anima_ctx* ctx, void* dst, const void* src, size_t bytes);
int anima_download(anima_ctx* ctx, void* dst, const void* src, size_t bytes);
/* Profiler (device.js:235-288): per-op CUDA-event timing, enabled by ANIMA_PROFILE=1. Writes a
 * text table into buf (NUL-terminated, truncated to cap). */
int anima_profile_report(anima_ctx* ctx, char* buf, size_t cap);
int anima_version(void);

/* ---------------------------------------------------------------- weights (weights.js, gemm.js) */
/* Decode 4-bit codes to their int8-grid values, bit-exact with tools/quant.py:179-180 and the
 * tile loader of app/gpu/gemm.js:141-158: grid = clamp(rne(cb[code] * fp8(s_rel)), -127, 127).
 * out: int8 [N, K]. */
int anima_unpack_w4(anima_ctx* ctx, const uint8_t* packed, const uint8_t* s_rel, const float* codebook, int N, int K,
                    int8_t* out);

/* ---------------------------------------------------------------- operators (ops.js) */
/* ops.linear (ops.js:48-66) for ConvRot weights: tcgen05 kind::i8 GEMM of the quantized rows x
 * with W, fused epilogue. W of kind I8 is used as stored. W of kind W4 (the reference's "w4" path,
 * app/gpu/gemm.js:141-158) stays packed in memory (0.5 byte per weight plus the fp8 group scales);
 * each call first decodes it to its int8 grid (the arithmetic of anima_unpack_w4, so the result is
 * bit-identical to unpacking once and passing kind I8) into a buffer the context owns (16 MiB or
 * the layer's N*K bytes, allocated on the first W4 call and grown outside stream capture only),
 * then runs the same GEMM on it. */
int anima_linear(anima_ctx* ctx, const anima_qact* x, const anima_weight* W, const anima_linear_opts* o);

/* runMatmul for "bf16"/"f32" weights (ops.js:14-33, gemm.js:81-127): C = epi(alpha A B^T),
 * A fp32 [M, lda], B bf16/f32 [N, ldb]; epilogue (+bias[n]) act, then store or C += gate*y.
 * Used for x_embedder, final layer, time conditioning and the LoRA down/up products. bf16 weights
 * with alpha 1, no activation and no gate, M >= 256, K and lda multiples of 8, ldc == N and 16-byte
 * aligned A, B and C run on the tensor cores with A split into two bf16 planes (as anima_conv3x3,
 * sharing its buffer; inside stream capture only when that buffer is already large enough); the
 * rest, and all fp32 weights, on a CUDA-core kernel with fp32 products. */
int anima_matmul(anima_ctx* ctx, int M, int N, int K, float alpha, const float* A, int lda, const anima_weight* B,
                 int act, float* C, int ldc, int accumulate, const float* gate, int gate_off);

/* LoRA down-projection for every side path of a linear at once (ops.js:78-79, the first GEMM of
 * loraDelta): T[m, j] = sum_k x[m, k] * A[j, k] with x the quantized rows the base GEMM consumes
 * and A the entries' (rotated) down matrices stacked [r, K] fp32; T fp32 [rows, ldt]. */
int anima_lora_down(anima_ctx* ctx, const anima_qact* x, const float* A, int r, float* T, int ldt);

/* ops.layernormMod (ops.js:129-137, kernels.js:95-145): y = LN(x)*(1+mod[scale_off+c]) +
 * mod[shift_off+c], optionally followed by the 256-point ConvRot Hadamard. out_dtype F32/BF16/F16. */
int anima_layernorm_mod(anima_ctx* ctx, const float* x, int rows, int cols, const float* mod, int shift_off,
                        int scale_off, float eps, int rotate, void* out, int out_dtype);
/* Same, fused with ConvRot and the per-token quantization a quantized linear consumes. */
int anima_layernorm_mod_quant(anima_ctx* ctx, const float* x, int rows, int cols, const float* mod, int shift_off,
                              int scale_off, float eps, const anima_qact* out);
/* ops.rotate (ops.js:38-44, kernels.js:359-388): y = x H per 256 group. in/out dtype F32/BF16/F16. */
int anima_rotate(anima_ctx* ctx, const void* x, int in_dtype, int rows, int cols, int ldx, void* y, int out_dtype);
/* ops.rotate fused with per-token quantization into anima_qact (input F32/BF16/F16). */
int anima_rotate_quant(anima_ctx* ctx, const void* x, int in_dtype, int rows, int cols, int ldx, const anima_qact* out);
/* Activation (GELU) then ConvRot then per-token quantization: the MLP hidden between layer1 (which
 * stores its pre-activation) and layer2 (dit.js:308-310, reference.py:242). act: ANIMA_ACT_NONE/GELU. */
int anima_act_rotate_quant(anima_ctx* ctx, const void* x, int in_dtype, int rows, int cols, int ldx, int act,
                           const anima_qact* out);
/* Per-token quantization without rotation (input already rotated). */
int anima_quant_rows(anima_ctx* ctx, const void* x, int in_dtype, int rows, int cols, int ldx, const anima_qact* out);
/* ops.rmsnorm (ops.js:111-117): y = x * rsqrt(mean(x^2) + eps) * w over rows of `cols`. */
int anima_rmsnorm(anima_ctx* ctx, const void* x, int in_dtype, int rows, int cols, const float* w, float eps, void* y,
                  int out_dtype);
/* ops.qkNormRope (ops.js:140-145, kernels.js:301-334), in place on qkv [L, ld] (dtype F32/BF16/F16). */
int anima_qk_norm_rope(anima_ctx* ctx, void* qkv, int dtype, int L, int H, int D, int ld, const float* qn,
                       const float* kn, const float* rope, int rope_rows, float eps);
/* ops.rope (ops.js:148-152, kernels.js:336-357), in place on x viewed as [L, H, D] at colOff. */
int anima_rope(anima_ctx* ctx, void* x, int dtype, int L, int H, int D, int row_stride, int col_off,
               const float* rope, int rope_rows);
/* ops.attention (ops.js:166-208, kernels.js:147-299): multi-head attention with fp32 softmax.
 * head_dim 128 with bf16/fp16 q/k/v (the DiT's attentions; the Qwen3 text encoder's, causal with
 * grouped k/v heads): the tcgen05 flash kernel. fp32 q/k/v with one wide head (head_dim a multiple
 * of 64, at least 2^20 scores: the VAE's d = 384 attention): tensor-core GEMMs around a row
 * softmax, with the fp32 scores materialised in a context buffer (Lq Lk 8 bytes plus the operand
 * planes, grown outside stream capture only). Everything else (head_dim 64, fp32 q/k/v, small
 * problems): a CUDA-core kernel over 32-key tiles in shared memory.
 * The stream-K schedule (see anima_ctx_set_attention_split) launches one CTA per SM and lets a CTA
 * wait, bounded at 2 s, for a partial result written by a lower-numbered CTA; it therefore needs
 * all of the device's SMs to be available to this kernel at once. Where other work can hold SMs
 * for long (MPS clients, green contexts, a long kernel on a concurrent stream), a wait can run out
 * and the call then reports ANIMA_ERR_DEVICE at anima_sync; set the split mode to 0 (whole units,
 * no waits between CTAs) on such hosts. */
int anima_attention(anima_ctx* ctx, const anima_attention_args* a);
/* anima_attention for callers that cannot call cudaMalloc (no reference counterpart): hosts whose
 * device memory belongs to another allocator or pool, or that must not allocate once running.
 * anima_attention allocates its stream-K workspace (20 MB) on first use; this entry point instead
 * uses a static device array in the library (21.6 MB: ready flags for up to 160 SMs, then one
 * 135 KB partial slot per SM), held by every GPU that loads the library until exit. Its first call
 * on a device looks up the array's address (cudaGetSymbolAddress, with that device current) and
 * clears the flags with a memset on the context's stream; make that first call before any stream
 * capture. Every launch leaves the flags at zero again. Same arguments, schedule and results as
 * anima_attention. Fails with ANIMA_ERR_ARG when the device has more SMs than the array has slots.
 * All calls share the array: calls on one device that overlap on the GPU (any context or stream)
 * race. */
int anima_attention_noalloc(anima_ctx* ctx, const anima_attention_args* a);
/* ops.elementwise (ops.js:154-160): op 0 copy, 1 add, 2 silu, 3 silu_mul; n fp32 elements. */
int anima_elementwise(anima_ctx* ctx, int op, const float* a, const float* b, float* y, long long n);
/* ops.zero (ops.js:89-93). */
int anima_zero(anima_ctx* ctx, void* p, size_t bytes);

/* ---------------------------------------------------------------- VAE decoder (vae.js) */
/* ops.conv3x3 / conv3x3Into (ops.js:97-109, the conv3 tiles of gemm.js): NHWC 3x3 convolution,
 * pad 1, of x fp32 [h * w, cin] with W bf16 OHWI [N, 9 cin] (+ W.bias); with up != 0 the input is
 * first upsampled 2x (nearest, the Resample of the Wan decoder). out fp32 [H * Wd, N] (H, Wd the
 * output size) = the result, or += it when accumulate != 0 (a residual). cin a multiple of 8.
 * Runs on the tensor cores with x split into two bf16 planes (hi + lo, about 16 significant bits;
 * fp32 accumulation), held in a buffer the context allocates on first use and grows, outside
 * stream capture only, to 4 bytes per input element (after the upsample). */
int anima_conv3x3(anima_ctx* ctx, const float* x, int h, int w, int cin, const anima_weight* W, int up, float* out,
                  int accumulate);
/* ops.channelNorm (ops.js:120-126, the Wan decoder's RMS_norm): y = x / max(||x||_2, 1e-12) *
 * sqrt(C) * gamma over each row of C channels, then SiLU when silu != 0; fp32. */
int anima_channel_norm(anima_ctx* ctx, const float* x, long long rows, int C, const float* gamma, int silu, float* y);

/* ---------------------------------------------------------------- model glue (dit.js, pipeline.js) */
/* patchify (dit.js:55-65): latent [B, 16, h, w] -> patches [B, (h/2)(w/2), 68] with the zero mask channel. */
int anima_patchify(anima_ctx* ctx, const float* latent, int B, int h, int w, float* patches);
/* unpatchify (dit.js:68-78): [B, (h/2)(w/2), 64] -> [B, 16, h, w]. */
int anima_unpatchify(anima_ctx* ctx, const float* o, int B, int h, int w, float* latent);
/* timestepEmbedding (dit.js:41-51) for B sigmas (device array): temb [B, 2048]. */
int anima_timestep_embedding(anima_ctx* ctx, const float* sigmas, int B, float* temb);
/* CFG combine + x0 prediction + Euler step (pipeline.js:260-269, samplers.js:109-117):
 *   v = v_uncond ? v_uncond + cfg (v - v_uncond) : v;  den = x - sigma v;
 *   x = (sigma_next == 0) ? den : (sigma_next/sigma) x + (1 - sigma_next/sigma) den.
 * den_out may be NULL. */
int anima_euler_step(anima_ctx* ctx, float* x, const float* v, const float* v_uncond, float cfg, float sigma,
                     float sigma_next, long long n, float* den_out);
/* Diagnostic with no counterpart in the reference: runs one bounded wait (the same as the
 * kernels' pipeline waits) on a barrier that is never released, so it gives up after timeout_us
 * (1 us .. 2 s), records "data wait timed out" in the device error word and returns; the next
 * anima_sync reports that error (ANIMA_ERR_DEVICE) and clears it, and the context stays usable.
 * result[0] = 1 if the wait completed (it should not), result[1] = the kernel's abort flag.
 * Exercises the failure path without a GPU fault. Synchronous. */
int anima_selftest_wait_timeout(anima_ctx* ctx, unsigned timeout_us, int* result);
/* The samplers' latent updates (samplers.js:104-218: axpby and the noise/derivative terms of
 * euler_a, dpmpp_2m and er_sde, and den = x - sigma v with CFG in pipeline.js:260-269):
 *   y[i] = c[0] x0[i] + c[1] x1[i] + c[2] x2[i] + c[3] x3[i] over n fp32 elements.
 * A NULL x_k drops its term; y may be any of the x_k (elementwise, in place). */
int anima_lincomb(anima_ctx* ctx, float* y, long long n, const float* x0, const float* x1, const float* x2,
                  const float* x3, const float* c);

/* ---------------------------------------------------------------- several GPUs of one node */
/* Peer memory for the sequence-parallel mode, where the ranks of one node split an image's token
 * rows and exchange self-attention keys/values (no reference counterpart: the reference runs on
 * one GPU). One process per GPU; buffers are shared with CUDA IPC, written by kernels over NVLink.
 *
 * anima_ipc_alloc: a plain device allocation of `bytes` on the context's device, zero-filled,
 *   and its 64-byte IPC handle (to hand to the other ranks, e.g. through torch.distributed).
 * anima_ipc_open: map another process's handle into this one (peer access enabled); returns the
 *   device address to use in this process. anima_ipc_close unmaps it; anima_ipc_free frees an
 *   anima_ipc_alloc allocation (after every other rank closed its mapping). */
int anima_ipc_alloc(anima_ctx* ctx, size_t bytes, void** ptr, unsigned char handle[64]);
int anima_ipc_open(anima_ctx* ctx, const unsigned char handle[64], void** ptr);
int anima_ipc_close(anima_ctx* ctx, void* ptr);
int anima_ipc_free(anima_ctx* ctx, void* ptr);

/* The ranks of one node, for anima_peer_barrier. flags[r] is rank r's flag array (world unsigned,
 * from anima_ipc_alloc, zeroed) as mapped in this process (this rank's own at flags[rank]);
 * counter is this rank's private barrier count (device memory, zero at start). */
typedef struct {
  int rank, world;         /* world <= 8 */
  unsigned* flags[8];
  unsigned* counter;
  unsigned timeout_us;     /* 0 = 2 s */
} anima_peer_group;

/* Device-side barrier of all ranks, in stream order: the kernel raises this rank's next epoch in
 * every rank's flags (system-scope release after a system fence, so this rank's earlier kernels'
 * writes to peer memory are visible first) and waits (acquire) until every rank has raised it.
 * Every rank must call it the same number of times. A wait that runs past the timeout records
 * "cross-GPU barrier timed out" in the device error word (reported by anima_sync) and returns;
 * nothing hangs. Safe inside CUDA graphs: the epoch lives in device memory. */
int anima_peer_barrier(anima_ctx* ctx, const anima_peer_group* g);

#ifdef __cplusplus
}
#endif
#endif /* ANIMA_B200_H */
