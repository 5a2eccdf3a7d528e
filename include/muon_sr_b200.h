/*
 * muon_sr_b200 -- C ABI of the B200 (sm_100a) optimizer-step engine.
 *
 * Every entry point takes plain device pointers, element counts and a CUDA stream
 * (cudaStream_t passed as an opaque handle), enqueues its kernels on that stream and
 * returns an msr_status. Nothing here allocates device memory: callers own every buffer
 * (parameters, gradients, optimizer states and the Newton-Schulz workspace, whose size
 * msr_ns_workspace_bytes reports). No entry point synchronises the stream except
 * msr_device_error.
 *
 * The reference (bab2min/muon_sr 0.1.2) is a Python package whose device work is a set of
 * Triton kernels plus torch.matmul; each entry point below replaces one of those launch
 * sites and cites it. Random seeds are the 64-bit Philox keys that the reference's Triton
 * kernels derive from their Python seed arguments; the Python layer of this package
 * computes them with the reference's formulas (muon_sr/triton_muon_sr.py:83-85).
 */
#ifndef MUON_SR_B200_H
#define MUON_SR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* msr_stream_t; /* a cudaStream_t; NULL is the legacy default stream */

enum msr_status {
  MSR_OK = 0,
  MSR_ERR_INVALID = 1,        /* bad argument: null pointer, negative size, bad shape */
  MSR_ERR_CUDA = 2,           /* a CUDA runtime call or kernel launch failed */
  MSR_ERR_UNSUPPORTED = 3,    /* valid request this build cannot run (e.g. not sm_100) */
  MSR_ERR_WORKSPACE = 4,      /* workspace smaller than msr_ns_workspace_bytes() */
  MSR_ERR_DEVICE_TIMEOUT = 5  /* a kernel gave up on a barrier wait (see msr_device_error) */
};

/* Version of this ABI (bumped on any signature change). */
int msr_abi_version(void);

/* Stochastic-rounding noise stream of every rounding kernel (process-wide; no counterpart
 * in the reference):
 *   MSR_SR_NOISE_REFERENCE (default) -- word 0 of Philox4x32-10 at the element offset
 *     truncated to 32 bits, one generator call per rounded value: the reference's bits.
 *   MSR_SR_NOISE_FAST -- one Philox4x32-10 call per 8 consecutive elements: element counter
 *     c uses 16-bit half (c & 1) of output word ((c >> 1) & 3) at counter (c >> 3), same
 *     keys. Each value is still rounded up with probability equal to its fractional part
 *     (unbiased stochastic rounding), but the bits differ from the reference's.
 *   MSR_SR_NOISE_NONE -- no stochastic rounding: every SR store rounds to the nearest bf16
 *     (ties to even) instead, as a plain fp32 -> bf16 cast would. A parity mode for checking
 *     the fp32 arithmetic of the updates without noise; not for training.
 * Returns MSR_ERR_INVALID for an unknown mode. */
enum msr_sr_noise { MSR_SR_NOISE_REFERENCE = 0, MSR_SR_NOISE_FAST = 1, MSR_SR_NOISE_NONE = 2 };
int msr_set_sr_noise(int mode);
/* The current mode (MSR_SR_NOISE_*). The Python layer applies the environment variable
 * MSR_SR_NOISE=reference|fast|none when it loads the library. */
int msr_get_sr_noise(void);
/* Static description of a status code. */
const char* msr_status_string(int status);
/* Detail message of the last failing call on the calling host thread ("" if none). */
const char* msr_last_error(void);
/* Synchronises `stream`, returns the device-side error code recorded by any kernel of
 * this library since the last clear (0 = none) and clears it when `clear` != 0. Codes: the
 * first wait that ran out of time, 0x101 / 0x102 / 0x103 for the GEMM's copy, MMA and
 * epilogue roles, 0x1FF for msr_test_wait_timeout. Every device-side wait of this library
 * is bounded (1 s); a kernel that gives up drains its own copies, frees its tensor memory
 * and returns, so the context stays usable. */
int msr_device_error(msr_stream_t stream, int clear);
/* Failure-detection test hook (no counterpart in the reference): launches one kernel that
 * waits, with the GEMM's bounded wait, on a barrier nothing arrives on and gives up after
 * `limit_ns` (at most 10 s), recording 0x1FF for msr_device_error. */
int msr_test_wait_timeout(uint64_t limit_ns, msr_stream_t stream);
/* Number of kernels this library has launched in this process (all threads, all devices). */
uint64_t msr_launch_count(void);
/* Caps the number of CTAs (one per SM) of the persistent GEMM kernels; 0 = one per SM (the
 * default). A caller that runs collectives concurrently with the optimizer step (e.g. the
 * sharded step's weight broadcasts) leaves SMs free for them this way. Process-wide. */
void msr_set_gemm_max_ctas(int max_ctas);
/* Selects the GEMM kernel of Newton-Schulz and msr_gemm_bf16: `enable` != 0 (the default)
 * runs 256 x 256 tiles on pairs of SMs (a 2-CTA cluster sharing each B tile), 0 runs
 * 128 x 256 tiles on single SMs. Both give the same results; process-wide. No counterpart
 * in the reference (its GEMMs are cuBLAS calls). */
void msr_set_gemm_pairs(int enable);
/* 1 if SM-pair tiles are selected (the default); the Python layer applies MSR_GEMM_PAIRS=0|1. */
int msr_get_gemm_pairs(void);

/* ---- Philox (test hook) ------------------------------------------------------------
 * out[i] = word 0 of Philox4x32-10 with counter ((ctr_base + i) mod 2^32, 0, 0, 0) and key
 * `key`: Triton's tl.randint(seed, offset) as muon_sr's kernels call it
 * (muon_sr/triton_muon_sr.py:44, muon_sr/triton_adamw.py:52). */
int msr_philox_fill(uint32_t* out, int64_t n, uint64_t ctr_base, uint64_t key, msr_stream_t stream);

/* ---- SR gradient accumulation ------------------------------------------------------
 * acc[i] <- SR_bf16(float(acc[i]) + float(grad[i])), counter i. With first != 0 the
 * accumulator is treated as zero and only written: acc[i] <- SR_bf16(0 + grad[i]), which is
 * grad[i] itself except that -0 becomes +0 (the reference zero-fills, then accumulates).
 * Replaces the _grad_accum_kernel launch of TritonSRAccumulator._accum_hook
 * (muon_sr/triton_adamw.py:206-229, launched at :259-265). */
int msr_grad_accum_bf16(void* acc, const void* grad, int64_t n, uint64_t key, int first, msr_stream_t stream);

/* ---- Muon momentum / Nesterov prepare ----------------------------------------------
 * Per entry, per element i < numel:
 *   new_buf = buf + one_minus_beta * (g - buf)
 *   upd     = nesterov ? g + beta * (new_buf - g) : new_buf
 *   momentum[i] <- SR_bf16(new_buf) with counter (ctr_base + i) mod 2^32
 *   update[i]   <- RNE_bf16(upd)
 * grad and update may alias (the reference prepares in place on its stacked workspace).
 * Replaces _muon_prepare_kernel launches (muon_sr/triton_muon_sr.py:18-50, launched at
 * :94-97 per parameter and :156-159 per shape stack, where ctr_base = index * numel). */
typedef struct msr_prepare_entry {
  const void* grad;    /* bf16[numel] */
  void* momentum;      /* bf16[numel], updated in place */
  void* update;        /* bf16[numel], output */
  int64_t numel;
  uint64_t ctr_base;
  uint64_t key;
} msr_prepare_entry;

int msr_muon_prepare(const msr_prepare_entry* entries, int count, float beta, float one_minus_beta,
                     int nesterov, msr_stream_t stream);

/* ---- Multicast weights (sharded steps; no counterpart in the single-device reference) ----
 * The weight-updating entries below (apply, AdamW, 8-bit AdamW) carry `param_mc`: NULL, or
 * the NVLink multicast address of `param` -- the same offset in a symmetric allocation that
 * every rank of the node maps and that is bound to one multicast object. With it, the kernel
 * stores the updated weight once through that address (multimem.st, 16-byte vectors) and
 * the NVSwitch writes it into every rank's replica, its own included: the update and the
 * weight all-gather are one kernel. The weight is still read from `param` (this rank's
 * replica). Requirements: `param_mc` 16-byte aligned like `param`, and when numel is odd the
 * element after the last one is padding nobody reads (a ragged end is stored in 4-byte
 * pairs). Readers on other ranks must be ordered after the writing kernel (a device barrier
 * across the ranks); each CTA ends its multicast stores with a system-scope fence. */

/* ---- Muon apply ----------------------------------------------------------------------
 * Per entry: param[i] <- SR_bf16(float(param[i]) * decay - lr * (float(update[i]) * scale)),
 * counter i, with decay = fp32(1 - lr * weight_decay) computed by the caller in double.
 * Replaces _muon_apply_kernel launches (muon_sr/triton_muon_sr.py:53-80, :105-113). */
typedef struct msr_apply_entry {
  void* param;         /* bf16[numel], updated in place */
  const void* update;  /* bf16[numel] (Newton-Schulz output) */
  int64_t numel;
  uint64_t key;
  float scale;         /* sqrt(max(1, rows/cols)) of the parameter's shape */
  float reserved;
  void* param_mc;      /* NULL or the multicast address of param (see above) */
} msr_apply_entry;

int msr_muon_apply(const msr_apply_entry* entries, int count, float lr, float decay, msr_stream_t stream);

/* ---- AdamW with stochastic rounding ------------------------------------------------
 * Per entry, per element:
 *   m = beta1*m + one_minus_beta1*g;  v = beta2*v + one_minus_beta2*g*g
 *   denom = sqrt(v)/bc2_sqrt + eps;  p = p*decay;  p = p - step_size*m/denom
 *   m, v, p <- SR_bf16 with keys key_m, key_v, key_p (the reference's seed, seed+1, seed+2)
 * step_size = fp32(lr / (1 - beta1^step)), bc2_sqrt = fp32(sqrt(1 - beta2^step)).
 * Replaces _adamw_kernel launches (muon_sr/triton_adamw.py:9-114). */
typedef struct msr_adamw_entry {
  void* param;
  const void* grad;
  void* exp_avg;
  void* exp_avg_sq;
  int64_t numel;
  uint64_t key_m, key_v, key_p;
  float step_size;
  float bc2_sqrt;
  void* param_mc;      /* NULL or the multicast address of param (see "Multicast weights") */
} msr_adamw_entry;

typedef struct msr_adamw_hparams {
  float beta1, one_minus_beta1, beta2, one_minus_beta2, eps, decay;
} msr_adamw_hparams;

int msr_adamw_sr(const msr_adamw_entry* entries, int count, const msr_adamw_hparams* hp,
                 msr_stream_t stream);

/* ---- Replayable launches (CUDA graphs) -------------------------------------------------
 * msr_muon_prepare_rec / msr_muon_apply_rec / msr_adamw_sr_rec launch the kernels of
 * msr_muon_prepare / msr_muon_apply / msr_adamw_sr, but the kernels read the launch's
 * scalars and its entry table from `record`, in device memory, instead of from the launch
 * parameters. A record (16-byte aligned) is the header struct below directly followed by
 * `count` entries. `entries` (host memory) must list the same tensors and sizes as the
 * record: it splits and sizes the launch and is validated as in the plain calls. A CUDA graph
 * captured around these calls replays with whatever the records hold when its kernels run,
 * so a caller moves a captured optimizer step to the next step -- new keys, bias
 * corrections, learning rates -- by rewriting the scalar fields of its records (e.g. with a
 * host-to-device copy captured at the start of the graph), without capturing again. The
 * pointers and sizes in a record must stay those of the capture. No counterpart in the
 * reference (its Triton launches take every scalar as a launch argument). */
typedef struct msr_prepare_record {
  float beta, one_minus_beta;
  int32_t nesterov;
  int32_t count;       /* entries that follow */
} msr_prepare_record;

typedef struct msr_apply_record {
  float lr, decay;
  int32_t count;
  int32_t reserved;
} msr_apply_record;

typedef struct msr_adamw_record {
  msr_adamw_hparams hp;
  int32_t count;
  int32_t reserved;
} msr_adamw_record;

int msr_muon_prepare_rec(const msr_prepare_entry* entries, int count, const void* record, msr_stream_t stream);
int msr_muon_apply_rec(const msr_apply_entry* entries, int count, const void* record, msr_stream_t stream);
int msr_adamw_sr_rec(const msr_adamw_entry* entries, int count, const void* record, msr_stream_t stream);

/* Gradient centralisation for TritonAdamW's `centralization` option: grad viewed as
 * [rows][cols] (rows = leading dim, or 1 for a vector), out = bf16_rne(g - c * mean_row)
 * with the row mean in fp32. One read of the gradient, one bf16 write (out must not
 * overlap grad). Replaces the torch ops of muon_sr/triton_adamw.py:179-187; the fp32 mean
 * is summed in a fixed order, which can differ from torch's reduction in its last bit. */
int msr_centralize_bf16(const void* grad, void* out, int64_t rows, int64_t cols, float centralization,
                        msr_stream_t stream);

/* ---- 8-bit blockwise AdamW -----------------------------------------------------------
 * One pass per tensor: dequantise (codebook x block absmax), Adam moments with the
 * non-finite-gradient mask, p' = (p - coef*m/(sqrt(v) + sqrt_bc2_eps)) * decay with SR
 * (key_p), then per block of block_size elements absmax and requantise with the 7-step
 * codebook search (quantized != 0), or SR bf16 moments (keys key_m, key_v) otherwise.
 * coef = fp32(fp32(lr)*sqrt(bc2)/bc1), sqrt_bc2_eps = fp32(sqrt(bc2))*fp32(eps).
 * Replaces _adamw_8bit_kernel launches (muon_sr/triton_adamw_8bit.py:56-99, :198-204). */
typedef struct msr_adamw8bit_entry {
  void* param;
  const void* grad;
  void* state1;        /* uint8 codes (quantized) or bf16 moments */
  void* state2;
  float* absmax1;      /* fp32[ceil(numel/block_size)] (quantized only) */
  float* absmax2;
  int64_t numel;
  uint64_t key_p, key_m, key_v;
  float coef;
  float sqrt_bc2_eps;
  int32_t quantized;
  int32_t reserved;
  void* param_mc;      /* NULL or the multicast address of param (see "Multicast weights") */
} msr_adamw8bit_entry;

typedef struct msr_adamw8bit_hparams {
  float beta1, one_minus_beta1, beta2, one_minus_beta2, decay;
  int32_t block_size;  /* power of two in [32, 4096] */
  /* Optional quantiser lookup tables for (qmap1, qmap2) in device memory, NULL to run the
   * reference's 7-step codebook walk. Layout (MSR_QT_* below): uint8 codes[3][MSR_QT_NB]
   * (signed map x >= 0, signed map x < 0, unsigned map) at offset 0, then float
   * thresholds[3][256] at offset MSR_QT_T_OFFSET. Bucket of |x| = clamp((bits(|x|) >> 15)
   * - MSR_QT_BASE, 0, NB - 1); code = codes[s][bucket], then +1 (x >= 0) or -1 (x < 0) if
   * |x| >= thresholds[s][code]. The Python layer (muon_sr_b200/quant_tables.py) builds and
   * verifies them against the walk. */
  const void* qtables;
} msr_adamw8bit_hparams;

#define MSR_QT_NB 7682
#define MSR_QT_BASE 24831
#define MSR_QT_T_OFFSET 23056
#define MSR_QT_BYTES (MSR_QT_T_OFFSET + 3 * 256 * 4)

int msr_adamw8bit(const msr_adamw8bit_entry* entries, int count, const float* qmap1,
                  const float* qmap2, const msr_adamw8bit_hparams* hp, msr_stream_t stream);

/* ---- Newton-Schulz ---------------------------------------------------------------------
 * out[b] = NS_steps(x[b]) for b < batch, x and out bf16 [batch, rows, cols] contiguous.
 * Quintic iteration (a, b, c) = (3.4445, -4.7750, 2.0315) on the wide orientation
 * (X^T when rows > cols), normalised by the Frobenius norm. Each step is three batched
 * tcgen05 GEMMs with fused epilogues: A = X X^T, B = c*(A A) + b*A, X' = B X + a*X.
 * mode MSR_NS_REFERENCE_ROUNDING rounds to bf16 exactly where the reference's torch ops
 * do -- X0 = bf16(x / bf16(bf16(||x||) + 1e-7)), A = bf16(acc),
 * B = bf16(bf16(b*A) + bf16(c*bf16(acc))), X' = bf16(bf16(a*X) + bf16(acc)) -- with
 * every rounding inside the GEMM epilogues. mode MSR_NS_FUSED_ROUNDING rounds once per
 * GEMM (alpha*acc + beta*C in fp32) and folds 1/(||x||+1e-7) into the first step; it is
 * closer to exact arithmetic but further from the reference's bits.
 * norm_sq, if given, holds ||x[b]||_F^2 (e.g. from msr_muon_prepare); otherwise it is
 * computed. out must not alias x.
 * Replaces _newton_schulz (muon_sr/muon_sr.py:82-98) with out_dtype=None, as called at
 * muon_sr/triton_muon_sr.py:119 and :166. */
enum msr_ns_mode { MSR_NS_REFERENCE_ROUNDING = 0, MSR_NS_FUSED_ROUNDING = 1 };

size_t msr_ns_workspace_bytes(int64_t batch, int64_t rows, int64_t cols);

int msr_newton_schulz_bf16(const void* x, void* out, int64_t batch, int64_t rows, int64_t cols,
                           int steps, int mode, const float* norm_sq, void* workspace,
                           size_t workspace_bytes, msr_stream_t stream);

/* ---- Newton-Schulz without a workspace (no counterpart in the reference) ---------------
 * For callers that cannot allocate device memory -- e.g. a plugin whose host program owns
 * every device allocation through its own pool and passes in only input and output
 * buffers, or a C / FFI caller with no device allocator -- this computes exactly what
 * msr_newton_schulz_bf16 computes, taking its scratch from a fixed 64 MiB area in the
 * library's own device memory instead of a workspace. It calls no cudaMalloc / cudaFree.
 * - Limit: requests with msr_ns_workspace_bytes(batch, rows, cols) > 64 MiB are rejected
 *   with MSR_ERR_WORKSPACE (e.g. up to a 2048 x 2048 matrix, or 4 of 1024 x 1024).
 * - Every GPU that loads the library holds the 64 MiB area until the process exits.
 * - The first call on a device looks up the area's address on that device; make that first
 *   call before any stream capture. The address is kept for the life of the process: after
 *   cudaDeviceReset (or anything else that destroys the device's primary context) it is
 *   stale, so do not call this function again in that process.
 * - All calls share the one area: calls that overlap on the GPU (other streams, other host
 *   threads without ordering) race and corrupt each other's results. Serialise them. */
int msr_newton_schulz_bf16_noalloc(const void* x, void* out, int64_t batch, int64_t rows,
                                   int64_t cols, int steps, int mode, const float* norm_sq,
                                   msr_stream_t stream);

/* ---- peer mappings for the sharded step (no counterpart in the single-device reference) --
 * The sharded optimizer (several ranks on one node, each updating the parameters it owns)
 * shares the updated bf16 weights with copy-engine peer copies over NVLink:
 * msr_ipc_export gives the 64-byte IPC handle of the device allocation holding ptr and ptr's
 * offset in it; msr_ipc_import maps such an allocation of another process (peer access is
 * enabled lazily); msr_ipc_close unmaps it; msr_copy_async enqueues one cudaMemcpyAsync
 * (peer-to-peer when the pointers live on different devices). Requires cudaMalloc'd
 * memory (not VMM / expandable segments). */
int msr_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out);
int msr_ipc_import(const void* handle, void** base_out);
int msr_ipc_close(void* base);
int msr_copy_async(void* dst, const void* src, size_t bytes, msr_stream_t stream);
/* Interprocess events ordering those copies: create (on the current device) and export a
 * 64-byte handle; open a peer's handle in the current device's context; record on / wait
 * from a stream; destroy. Events are opaque cudaEvent_t handles. */
int msr_ipc_event_create(void** event_out, void* handle_out);
int msr_ipc_event_open(const void* handle, void** event_out);
int msr_event_record(void* event, msr_stream_t stream);
int msr_stream_wait_event(msr_stream_t stream, void* event);
int msr_event_destroy(void* event);

/* ---- batched bf16 GEMM with the Newton-Schulz epilogue (test hook) --------------------
 * d[b] = alpha_b * (A[b] x B[b]^T) + beta_b * c[b] on the tensor cores, bf16 in/out,
 * fp32 accumulate. A is [batch, M, K] (a_mn_major = 0) or [batch, K, M] (1); B is
 * [batch, N, K] (b_mn_major = 0) or [batch, K, N] (1); c, d are [batch, M, N]; c may be
 * NULL. alpha_b = alpha * s^alpha_pow, beta_b = beta * s^beta_pow with s = scale[b]
 * (scale may be NULL). flags: MSR_GEMM_REFERENCE_ROUNDING makes the epilogue compute
 * bf16(bf16(beta*c) + bf16(alpha*bf16(acc))) (the reference's op-by-op rounding; no scale);
 * MSR_GEMM_SYMMETRIC (M == N, product known to be symmetric, e.g. A A^T) computes only the
 * tiles touching the upper triangle and mirror-writes the rest.
 * Rows of every operand must be a multiple of 16 bytes. */
enum msr_gemm_flags { MSR_GEMM_REFERENCE_ROUNDING = 1, MSR_GEMM_SYMMETRIC = 2 };

int msr_gemm_bf16(const void* a, int a_mn_major, const void* b, int b_mn_major, const void* c,
                  void* d, int64_t batch, int64_t M, int64_t N, int64_t K, float alpha, float beta,
                  const float* scale, int alpha_pow, int beta_pow, int flags, msr_stream_t stream);

/* Test hook, host only (no GPU needed): the GEMM kernels' tile schedule. Sets *num_tiles to
 * the number of output tiles a launch of this shape runs (`pairs`: 256 x 256 SM-pair tiles,
 * else 128 x 256; `symmetric`: only tiles touching the upper triangle, M == N) and, if `out`
 * holds 3 * num_tiles values, writes (matrix, first row, first column) of each linear tile
 * index in the order the persistent kernels take them -- the same decoding the kernels run. */
int msr_gemm_tile_map(int64_t M, int64_t N, int64_t batch, int symmetric, int pairs, int64_t* out,
                      int64_t capacity, int64_t* num_tiles);

#ifdef __cplusplus
}
#endif

#endif /* MUON_SR_B200_H */
