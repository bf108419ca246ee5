/*
 * lowbit.h -- C ABI of the B200 low-bit quantized-linear library (liblowbit.so).
 *
 * Plain pointers, sizes and a CUDA stream passed as `void*`.  Every entry point
 * returns an lb_status and never aborts.  All device buffers belong to the caller;
 * the library allocates no device memory (scratch is a caller-provided workspace
 * sized by the matching *_workspace_bytes query, 16-byte aligned and zero-filled once
 * before its first use -- kernels that keep arrival counters there leave them at zero
 * again).  A workspace serves one stream at a time.  Outputs must not alias inputs.
 * Work is stream-ordered and asynchronous unless a comment says otherwise.
 *
 * Packed formats are the reference's canonical bytes (torch_npu_lowbit.py):
 *   LB_FMT_INT4 / LB_FMT_NF4: two 4-bit codes per byte, even flat element in the
 *     low nibble, flattened row-major over [N,K], odd count padded with a zero
 *     high nibble (pack_codes, torch_npu_lowbit.py:24-30).  INT4 is symmetric
 *     two's complement (decoded ((c ^ 8) - 8)); NF4 indexes the 16-entry codebook.
 *   LB_FMT_INT8: one signed byte per element, row-major [N,K].
 *   LB_FMT_FP16: dense fp16 weights [N,K] (unquantized projections, tied LM head).
 *   scales: fp16 [N, K/group] row-major (per-row when group == K).
 * fp16 values are passed as uint16_t bit patterns.
 */
#ifndef LOWBIT_H_
#define LOWBIT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum lb_format { LB_FMT_INT4 = 0, LB_FMT_NF4 = 1, LB_FMT_INT8 = 2, LB_FMT_FP16 = 3 };

enum lb_status {
  LB_OK = 0,
  LB_ERR_INVALID_ARGUMENT = 1, /* bad shape / group / pointer / alignment  (Python: ValueError) */
  LB_ERR_UNSUPPORTED = 2,      /* valid request this build does not implement */
  LB_ERR_CUDA = 3,             /* a CUDA runtime call or launch failed       (Python: RuntimeError) */
  LB_ERR_NONFINITE = 4,        /* quantize: a weight is NaN/Inf ('Nonfinite weights cannot be quantized') */
  LB_ERR_SCALE_OVERFLOW = 5,   /* quantize: absmax/limit > fp16 max ('Weight scale overflows FP16') */
  LB_ERR_WORKSPACE = 6,        /* workspace missing or smaller than the query returned */
  LB_ERR_ALIAS = 7,            /* an output overlaps an input */
  LB_ERR_INJECTED = 8,         /* host-side fault injection (LOWBIT_INJECT_FAULT) */
  LB_ERR_TIMEOUT = 9           /* a bounded device-side wait gave up (error flag set, kernel returned) */
};

enum lb_path { LB_PATH_AUTO = 0, LB_PATH_GEMV = 1, LB_PATH_TC = 2, LB_PATH_GENERIC = 3 };

/* Human-readable text for a status code (static storage). */
const char *lb_status_string(int status);
/* ABI version, bumped on any signature change. */
int lb_abi_version(void);
/* The cudaError_t of the last LB_ERR_CUDA on this host thread (0 if none). */
int lb_last_cuda_error(void);
/* Host-side fault injection for tests: the next `count` calls of entry point `entry`
 * ("*" = any) return LB_ERR_INJECTED before launching anything.  No device fault is
 * ever produced.  (Replaces the driver-failure quarantine paths of backend.cpp:287-293
 * as the way failure handling is exercised.) */
int lb_inject_fault(const char *entry, int count);
/* SYNCHRONOUS: read the device-side status word at the start of a linear workspace
 * (LB_OK, or LB_ERR_TIMEOUT if a bounded device-side wait of a kernel that used it gave
 * up: the tensor-core GEMM's pipeline waits, or the decode GEMV's wait for the correction
 * projection computed inside the same launch).  No reference counterpart: the reference's
 * submissions are synchronous and report driver errors per call (backend.cpp:287-293). */
int lb_workspace_status(const void *workspace, void *stream);
/* SYNCHRONOUS: lb_workspace_status, and when the word is set, zero the workspace header
 * (status word and arrival counters; arrivals may have landed after a counter was reset)
 * so that the next call starts clean.  Returns the status read. */
int lb_workspace_check(void *workspace, size_t workspace_bytes, void *stream);
/* Test hook, no reference counterpart: the decode GEMV's wait for its in-launch
 * correction projection gives up after `wait_cycles` SM clock cycles (<= 0: the default,
 * about 2 s) and, with `missing_arrivals` > 0, waits for that many arrivals more than any
 * launch makes, so that the wait runs out.  The kernel then records LB_ERR_TIMEOUT and
 * returns; nothing faults.  Process-wide; call with (0, 0) to restore. */
int lb_test_wait_override(long long wait_cycles, int missing_arrivals);

/*
 * Quantize + pack on the GPU.  Replaces quantize_weight (torch_npu_lowbit.py:78-105):
 * symmetric per-group absmax, scale = fp16(max(absmax/limit, 2^-24)) with limit
 * 7 / 1 / 127, RTN-even codes (INT4/INT8) or NF4 midpoint search (searchsorted
 * side='left').  Bit-exact with the reference.  weight_dtype: 0 = fp32, 1 = fp16.
 * SYNCHRONOUS: waits for `stream` and returns LB_ERR_NONFINITE or
 * LB_ERR_SCALE_OVERFLOW exactly where the reference raises ValueError.
 */
size_t lb_quantize_workspace_bytes(void);
int lb_quantize_pack(int fmt, int group, const void *weight, int weight_dtype, int n, int k,
                     uint8_t *codes, uint16_t *scales, void *workspace, size_t workspace_bytes,
                     void *stream);

/*
 * fp16 dequantization on the GPU.  Replaces PackedWeight.dequantize
 * (torch_npu_lowbit.py:67-75): out = rn16(code_value_fp16 * scale_fp16); bit-exact.
 */
int lb_dequantize(int fmt, int group, int n, int k, const uint8_t *codes, const uint16_t *scales,
                  uint16_t *out, void *stream);

/*
 * y[M,N] = x[M,K] . deq(W)[N,K]^T (+ bias) (+ rank-r correction), fp16 in / out.
 * Replaces QuantizedLinear.forward (torch_npu_lowbit.py:339-360, which submits
 * through npu._run -> backend.cpp:253-295 -> graphinfer_session_infer) and the
 * per-projection linear of FrozenSmolLayer (torch_npu_smollm.py:150-164, :237-259).
 * Staging follows the reference CPU path: y_q = half(x . W^T) with fp32 (fp64 for
 * per-row INT8) accumulation; y = half(y_q + bias); z = half(x . V^T);
 * delta = half(z . U^T); y = half(y + delta).
 * down = V [rank, K], up = U [N, rank] (fp16, LowRankCorrection.tensors()), or NULL.
 * codes = packed bytes as above (fp16 weights for LB_FMT_FP16); scales NULL for FP16.
 */
size_t lb_linear_workspace_bytes(int fmt, int group, int m, int n, int k, int rank);
int lb_linear(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
              const uint16_t *scales, const uint16_t *down, const uint16_t *up, int rank,
              const uint16_t *bias, uint16_t *y, void *workspace, size_t workspace_bytes,
              void *stream);
/* Same as lb_linear with an explicit kernel family (enum lb_path) for tests/benchmarks. */
int lb_linear_path(int path, int fmt, int group, int m, int n, int k, const uint16_t *x,
                   const uint8_t *codes, const uint16_t *scales, const uint16_t *down,
                   const uint16_t *up, int rank, const uint16_t *bias, uint16_t *y,
                   void *workspace, size_t workspace_bytes, void *stream);
/* Which kernel family lb_linear would choose for this problem (enum lb_path). */
int lb_linear_select(int fmt, int group, int m, int n, int k, int rank);

/* Several linears that read the same activations, as one decode GEMV launch (M <= 64).
 * No reference counterpart: the reference runs q/k/v (and gate/up) as separate
 * QuantizedLinear calls (torch_npu_smollm.py:170-173, :187-188).  The caller stacks the
 * packed rows (codes, scales, bias) of the linears, which must share format and group,
 * and their corrections as one block-diagonal correction of the summed rank (<= 128):
 * down = [V_1; V_2; ...] ([rank, K]), up [N, rank] with each linear's U in its own
 * column block and zeros elsewhere, so every output equals the separate call's
 * staging exactly.  z (optional, [M, rank rounded up to 32], zero past the rank) is the
 * correction projection already computed by lb_rmsnorm_project / lb_silu_mul_project;
 * it replaces down.  residual (optional, [M, N]) is added last, y = half(y + residual):
 * the residual add of torch_npu_smollm.py:192 fused into the down projection.
 * Workspace: lb_linear_workspace_bytes(fmt, group, m, n, k, rank).  LB_ERR_UNSUPPORTED
 * when the problem is not a decode GEMV (M > 64, unaligned rows or pointers). */
int lb_linear_stacked(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                      const uint16_t *scales, const uint16_t *down, const uint16_t *up,
                      const uint16_t *z, int rank, const uint16_t *bias, const uint16_t *residual,
                      uint16_t *y, void *workspace, size_t workspace_bytes, void *stream);

/*
 * Allocation-free decode GEMV.  No counterpart in the reference (its linear runs inside
 * an NPU graph session that owns all of its buffers).
 *
 * For callers that cannot provide a workspace -- a host application linking this
 * library whose device memory belongs to an allocator it may not call, or a
 * latency-critical thread where a first cudaMalloc would block -- this is lb_linear
 * restricted to the decode GEMV (M <= 64, 16-byte aligned x / codes / y / factors).
 * Its scratch (correction projection, split-K partials, arrival counters) is one fixed
 * array of LB_NOALLOC_SCRATCH_BYTES compiled into the library; every GPU that loads the
 * library holds it until the process exits.  The call allocates nothing; the caller
 * still passes every input and the output.
 *   - The first call on a device looks up the array's device address for that device
 *     (the device that is current); make that first call before any stream capture.
 *   - Problems whose scratch would not fit return LB_ERR_WORKSPACE; other M return
 *     LB_ERR_UNSUPPORTED (use lb_linear with a workspace).
 *   - All calls on a device share the array: calls that can overlap on the GPU (for
 *     example on two streams without ordering between them) race and must not be made.
 *   - Each call clears the array's arrival counters and status word first; read the
 *     status with lb_noalloc_status.  An output overlapping an input is LB_ERR_ALIAS.
 */
#define LB_NOALLOC_SCRATCH_BYTES (4u << 20)
int lb_linear_gemv_noalloc(int fmt, int group, int m, int n, int k, const uint16_t *x,
                           const uint8_t *codes, const uint16_t *scales, const uint16_t *down,
                           const uint16_t *up, int rank, const uint16_t *bias, uint16_t *y,
                           void *stream);
/* SYNCHRONOUS: the status word the last lb_linear_gemv_noalloc call on the current
 * device left in the fixed array -- LB_OK, or LB_ERR_TIMEOUT when its bounded wait for
 * the correction projection gave up (its y is then not valid).  A set word is cleared
 * with the array's arrival counters.  Like lb_linear_gemv_noalloc, it allocates nothing. */
int lb_noalloc_status(void *stream);

/*
 * SmolLM decoder ops around the projections (torch_npu_smollm.py:142-193 staging,
 * torch_npu_smollm_io.py:45-61).  All fp16, row-major, stream-ordered.
 */
/* out = half(half(v * rsqrt(mean(v^2) + eps)) * gamma), v = float(x) (+ float(residual)
 * first, stored back to residual_out as half when non-NULL): torch_npu_smollm.py:166-168. */
int lb_rmsnorm(const uint16_t *x, const uint16_t *residual, uint16_t *residual_out,
               const uint16_t *gamma, uint16_t *out, int rows, int dim, float eps, void *stream);
/* In-place RoPE on q [T, heads, hd] and k [T, kv_heads, hd] with per-token positions:
 * v = half(half(v*cos) + half(rotate_half(v)*sin)) (torch_npu_smollm.py:174-177).
 * cos/sin tables are [table_rows, hd]; a token whose position is outside the table is
 * left unrotated. */
int lb_rope(uint16_t *q, uint16_t *k, const int32_t *positions, const uint16_t *cos_table,
            const uint16_t *sin_table, int table_rows, int tokens, int heads, int kv_heads,
            int head_dim, int q_stride, int k_stride, void *stream);
/* Append k/v rows [B, kv_heads, hd] into caches [B, kv_heads, max_pos, hd] at position
 * lengths[b] (the KV Select of torch_npu_smollm.py:288-292). */
int lb_kv_append(const uint16_t *k, const uint16_t *v, int kv_stride, uint16_t *k_cache,
                 uint16_t *v_cache, const int32_t *lengths, int batch, int kv_heads, int head_dim,
                 int max_pos, void *stream);
/* One-query GQA attention over the cache (torch_npu_smollm.py:178-182, the KV Select and
 * attention of :262-301): s = half(half(q.k) * scale), softmax in fp32 as an online
 * (running max / sum) pass, out = half(p . v) -- the reference rounds p to fp16 before
 * p . v, here p stays fp32.  Attends positions 0..lengths[b] (inclusive).  out
 * [B, heads*hd].  When batch x kv_heads gives too few CTAs, the positions of each
 * (sequence, kv head) are split across CTAs and merged in split order (deterministic);
 * the splits need `workspace` (lb_attention_workspace_bytes; it may be the same buffer
 * as a linear workspace on the same stream -- the arrival counters are shared and left at
 * zero).  A NULL or smaller workspace only reduces the splits. */
int lb_attention_decode(const uint16_t *q, int q_stride, const uint16_t *k_cache,
                        const uint16_t *v_cache, const int32_t *lengths, uint16_t *out, int batch,
                        int heads, int kv_heads, int head_dim, int max_pos, float scale,
                        void *workspace, size_t workspace_bytes, void *stream);
size_t lb_attention_workspace_bytes(int batch, int heads, int max_pos);
/* lb_rope of this step's q and k + lb_kv_append + lb_attention_decode as one launch
 * (torch_npu_smollm.py:174-182, :288-292).  No single reference call: the attention CTA
 * of (b, kv head) rotates and appends that head's new k row (and copies v) at position
 * lengths[b], then rotates q while loading it; same fp16 staging as the three calls.
 * k_new / v_new: [B, kv_stride] rows (column blocks of one q|k|v buffer allowed); q is
 * read, not written.  Positions at or past table_rows are attended unrotated.  Workspace
 * as for lb_attention_decode. */
int lb_attention_decode_rope(const uint16_t *q, int q_stride, const uint16_t *k_new,
                             const uint16_t *v_new, int kv_stride, const uint16_t *cos_table,
                             const uint16_t *sin_table, int table_rows, uint16_t *k_cache,
                             uint16_t *v_cache, const int32_t *lengths, uint16_t *out, int batch,
                             int heads, int kv_heads, int head_dim, int max_pos, float scale,
                             void *workspace, size_t workspace_bytes, void *stream);
/* h = half(half(silu(float(gate))) * up)  (torch_npu_smollm.py:189-190); gate/up may be
 * column blocks of one [rows, 2F] buffer (row stride in elements). */
int lb_silu_mul(const uint16_t *gate, const uint16_t *up, int in_stride, uint16_t *out, int rows,
                int cols, void *stream);
/* lb_rmsnorm / lb_silu_mul fused with the correction projection of the linear that
 * consumes their output: z[r, c] = half(sum_k out[r, k] down[c, k]) for c < rank, zero
 * up to the row stride (rank rounded up to 32).  No single reference call: the
 * reference computes x V^T inside each corrected linear (torch_npu_smollm.py:160-163);
 * the value is the same projection of the same fp16 row.  down / z null: plain op. */
int lb_rmsnorm_project(const uint16_t *x, const uint16_t *residual, uint16_t *residual_out,
                       const uint16_t *gamma, uint16_t *out, int rows, int dim, float eps,
                       const uint16_t *down, int rank, uint16_t *z, void *stream);
int lb_silu_mul_project(const uint16_t *gate, const uint16_t *up, int in_stride, uint16_t *out,
                        int rows, int cols, const uint16_t *down, int rank, uint16_t *z,
                        void *stream);
/* out[r] = half(a[r] + b[r]) elementwise (residual adds, torch_npu_smollm.py:184,192). */
int lb_add(const uint16_t *a, const uint16_t *b, uint16_t *out, int64_t count, void *stream);
/* rows of a fp16 table gathered by int64 ids (torch_npu_smollm_io.py:45-50). */
int lb_embed(const int64_t *ids, const uint16_t *table, uint16_t *out, int64_t tokens, int dim,
             int64_t vocab, void *stream);
/* Greedy argmax over fp16 logits rows (first index on ties, as torch.argmax). */
int lb_argmax(const uint16_t *logits, int rows, int vocab, int64_t *out, void *workspace,
              size_t workspace_bytes, void *stream);
size_t lb_argmax_workspace_bytes(int rows, int vocab);

#ifdef __cplusplus
}
#endif
#endif /* LOWBIT_H_ */
