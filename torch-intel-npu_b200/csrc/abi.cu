// The C ABI of liblowbit.so (declared in include/lowbit.h): host-side validation that
// mirrors the reference's ValueError checks, path selection, workspace carving, status
// codes and host-side fault injection.  No entry point allocates device memory.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

namespace lowbit_host {
// quantize.cu
cudaError_t launch_quantize(int fmt, int group, const void *w, int dtype, int n, int k, uint8_t *codes,
                            uint16_t *scales, int *flags, cudaStream_t stream);
cudaError_t launch_dequantize(int fmt, int group, int n, int k, const uint8_t *codes, const uint16_t *scales,
                              uint16_t *out, cudaStream_t stream);
// gemv.cu
bool gemv_supported(int fmt, int group, int m, int n, int k);
cudaError_t launch_lowrank_project(int m, int k, int rank, int zs, const uint16_t *x, const uint16_t *v, uint16_t *z,
                                   cudaStream_t st);
cudaError_t launch_gemv(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                        const uint16_t *scales, const uint16_t *z, int zs, const uint16_t *up, int rank,
                        const uint16_t *bias, const uint16_t *resid, uint16_t *y, void *scratch, int *counters,
                        cudaStream_t st);
size_t gemv_workspace_bytes(int fmt, int m, int n, int k);
cudaError_t launch_gemv_fused_z(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                                const uint16_t *scales, const uint16_t *down, const uint16_t *up, int rank,
                                const uint16_t *bias, uint16_t *y, void *scratch, int *counters, float *zpart,
                                int *err, cudaStream_t st, bool *fused);
size_t gemv_fused_zpart_bytes(int m);
void set_wait_override(long long cycles, int missing);
cudaError_t launch_linear_generic(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                                  const uint16_t *scales, const uint16_t *z, const uint16_t *up, int rank,
                                  const uint16_t *bias, uint16_t *y, cudaStream_t st);
// tc_gemm.cu
bool tc_supported(int fmt, int group, int m, int n, int k, int rank);
size_t tc_partial_bytes(int m, int n, int k);
cudaError_t launch_tc(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                      const uint16_t *scales, const uint16_t *z, const uint16_t *up, int rank, const uint16_t *bias,
                      uint16_t *y, int ldy, float *partial, int *counters, int *err, cudaStream_t st);
// decoder_ops.cu
cudaError_t launch_rmsnorm(const uint16_t *x, const uint16_t *res, uint16_t *res_out, const uint16_t *gamma,
                           uint16_t *out, int rows, int dim, float eps, cudaStream_t st);
cudaError_t launch_rope(uint16_t *q, uint16_t *k, const int32_t *pos, const uint16_t *cos_t, const uint16_t *sin_t,
                        int table_rows, int tokens, int heads, int kvh, int hd, int q_stride, int k_stride,
                        cudaStream_t st);
cudaError_t launch_kv_append(const uint16_t *k, const uint16_t *v, int kv_stride, uint16_t *kc, uint16_t *vc,
                             const int32_t *lengths, int batch, int kvh, int hd, int max_pos, cudaStream_t st);
size_t attention_scratch_bytes(int batch, int heads, int splits);
cudaError_t launch_row_project(int mode, const uint16_t *x, const uint16_t *res, uint16_t *res_out,
                               const uint16_t *gamma, uint16_t *out, int rows, int dim, int in_stride, float eps,
                               const uint16_t *v, int rank, uint16_t *z, cudaStream_t st);
cudaError_t launch_attention_decode_rope(const uint16_t *q, int q_stride, const uint16_t *k_new, const uint16_t *v_new,
                                         int kv_stride, const uint16_t *cos_t, const uint16_t *sin_t, int table_rows,
                                         uint16_t *kc, uint16_t *vc, const int32_t *lengths, uint16_t *out, int batch,
                                         int heads, int kvh, int hd, int max_pos, float scale, int *counters,
                                         void *scratch, size_t scratch_bytes, cudaStream_t st);
cudaError_t launch_attention_decode(const uint16_t *q, int q_stride, const uint16_t *kc, const uint16_t *vc,
                                    const int32_t *lengths, uint16_t *out, int batch, int heads, int kvh, int hd,
                                    int max_pos, float scale, int *counters, void *scratch, size_t scratch_bytes,
                                    cudaStream_t st);
cudaError_t launch_silu_mul(const uint16_t *gate, const uint16_t *up, int in_stride, uint16_t *out, int rows, int cols,
                            cudaStream_t st);
cudaError_t launch_add(const uint16_t *a, const uint16_t *b, uint16_t *out, int64_t count, cudaStream_t st);
cudaError_t launch_embed(const int64_t *ids, const uint16_t *table, uint16_t *out, int64_t tokens, int dim,
                         int64_t vocab, cudaStream_t st);
cudaError_t launch_argmax(const uint16_t *logits, int rows, int vocab, int64_t *out, cudaStream_t st);

bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char *s = getenv("LOWBIT_PDL");
    v = (s && s[0] == '0') ? 0 : 1;
  }
  return v == 1;
}
}  // namespace lowbit_host

using namespace lowbit_host;

namespace lowbit_host {
namespace {
// Host-side fault injection: the next `count` calls of entry `name` fail with
// LB_ERR_INJECTED before launching anything (no device fault is ever produced).
std::mutex g_inject_mu;
std::string g_inject_name;
std::atomic<int> g_inject_count{0};
}  // namespace

bool injected(const char *entry) {
  if (g_inject_count.load(std::memory_order_relaxed) <= 0) return false;
  std::lock_guard<std::mutex> lk(g_inject_mu);
  if (g_inject_count.load() <= 0) return false;
  if (g_inject_name != "*" && g_inject_name != entry) return false;
  g_inject_count.fetch_sub(1);
  return true;
}

bool overlaps(const void *a, size_t na, const void *b, size_t nb) {
  if (!a || !b || !na || !nb) return false;
  const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  return x < y + nb && y < x + na;
}

size_t code_bytes(int fmt, int64_t n, int64_t k) {
  const int64_t c = n * k;
  if (fmt == LB_FMT_INT8) return size_t(c);
  if (fmt == LB_FMT_FP16) return size_t(c) * 2;
  return size_t((c + 1) / 2);
}

int linear_alias_status(int fmt, int group, int m, int n, int k, const void *x, const void *codes, const void *scales,
                        const void *down, const void *up, int rank, const void *bias, const void *y) {
  const size_t yb = size_t(m) * n * 2;
  if (overlaps(y, yb, x, size_t(m) * k * 2) || overlaps(y, yb, codes, code_bytes(fmt, n, k)) ||
      (scales && overlaps(y, yb, scales, size_t(n) * (k / group) * 2)) ||
      (bias && overlaps(y, yb, bias, size_t(n) * 2)) || (down && overlaps(y, yb, down, size_t(rank) * k * 2)) ||
      (up && overlaps(y, yb, up, size_t(n) * rank * 2)))
    return LB_ERR_ALIAS;
  return LB_OK;
}
}  // namespace lowbit_host

namespace {
thread_local int g_last_cuda_error = 0;

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return LB_OK;
  g_last_cuda_error = int(e);
  return LB_ERR_CUDA;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool valid_format(int fmt) { return fmt == LB_FMT_INT4 || fmt == LB_FMT_NF4 || fmt == LB_FMT_INT8 || fmt == LB_FMT_FP16; }

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Workspace header: [0, 256) status word; [256, 256 + 16 KiB) GEMV arrival counters.
// Both sit at fixed offsets, so whatever shape a call has, the counters it relies on
// are the ones the previous call left at zero.
constexpr size_t kCounterOffset = 256;
constexpr size_t kHeader = 256 + 4096 * sizeof(int);

int select_path(int fmt, int group, int m, int n, int k, int rank) {
  // fp16 weights (the tied LM head) from 16 activation rows on: no dequant stands between the
  // TMA-loaded tile and the tensor cores, and the tcgen05 kernel wins by 1.6-5x (measured on
  // B200, 49152 x 960 / 2048 at 16-64 rows: 65 -> 41, 146 -> 42, 130 -> 26 us)
  if (fmt == LB_FMT_FP16 && m >= 16 && n >= 4096 && tc_supported(fmt, group, m, n, k, rank)) return LB_PATH_TC;
  if (gemv_supported(fmt, group, m, n, k)) return LB_PATH_GEMV;
  if (tc_supported(fmt, group, m, n, k, rank)) return LB_PATH_TC;
  return LB_PATH_GENERIC;
}

// z holds rank rounded up to 32 columns per activation row (32 for every lb_linear call),
// or the fp32 K-slice partials of a projection fused into the decode GEMV.
size_t z_bytes(int m, int rank) {
  return rank > 0 ? align256(std::max(size_t(m) * ((rank + 31) / 32 * 32) * 2, gemv_fused_zpart_bytes(m))) : 0;
}

// The z projection of a tcgen05 call: mma.sync tiles up to 16384 activation rows (a rank-32
// "weight" tile leaves three quarters of a tcgen05 tile empty, and the launch is short),
// the tcgen05 kernel above (measured on B200: 2048 and 8192 rows faster on mma.sync,
// 65536 rows faster on tcgen05).  LOWBIT_Z_TC=0 / 1 forces either (comparison).
bool z_on_tc(int m, int k, int rank) {
  static const char *env = getenv("LOWBIT_Z_TC");
  const bool tc = env ? env[0] == '1' : m > 16384;
  return tc && m > 32 && tc_supported(LB_FMT_FP16, k, m, rank, k, 0);
}

size_t linear_ws(int path, int fmt, int group, int m, int n, int k, int rank) {
  size_t b = kHeader + z_bytes(m, rank);
  if (path == LB_PATH_GEMV && gemv_supported(fmt, group, m, n, k)) b += align256(gemv_workspace_bytes(fmt, m, n, k));
  if (path == LB_PATH_TC && tc_supported(fmt, group, m, n, k, rank)) {
    b += align256(tc_partial_bytes(m, n, k));
    if (rank > 0 && z_on_tc(m, k, rank)) b += align256(tc_partial_bytes(m, rank, k));
  }
  return b;
}

int validate_linear(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                    const uint16_t *scales, const uint16_t *down, const uint16_t *up, int rank, const uint16_t *y) {
  if (!valid_format(fmt) || m < 1 || n < 1 || k < 1 || !x || !codes || !y) return LB_ERR_INVALID_ARGUMENT;
  if (fmt != LB_FMT_FP16 && (!scales || group < 1 || group > k || k % group)) return LB_ERR_INVALID_ARGUMENT;
  if ((down == nullptr) != (up == nullptr)) return LB_ERR_INVALID_ARGUMENT;
  if (down && (rank < 1 || rank > 32 || rank > n || rank > k)) return LB_ERR_INVALID_ARGUMENT;
  if (int64_t(m) * k > (int64_t(1) << 40) || int64_t(n) * k > (int64_t(1) << 40)) return LB_ERR_INVALID_ARGUMENT;
  return LB_OK;
}
}  // namespace

extern "C" {

const char *lb_status_string(int s) {
  switch (s) {
    case LB_OK: return "ok";
    case LB_ERR_INVALID_ARGUMENT: return "invalid argument";
    case LB_ERR_UNSUPPORTED: return "unsupported";
    case LB_ERR_CUDA: return "CUDA error";
    case LB_ERR_NONFINITE: return "Nonfinite weights cannot be quantized";
    case LB_ERR_SCALE_OVERFLOW: return "Weight scale overflows FP16";
    case LB_ERR_WORKSPACE: return "workspace missing or too small";
    case LB_ERR_ALIAS: return "output aliases an input";
    case LB_ERR_INJECTED: return "injected fault";
    case LB_ERR_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

int lb_abi_version(void) { return 2; }

int lb_last_cuda_error(void) { return g_last_cuda_error; }

int lb_inject_fault(const char *entry, int count) {
  std::lock_guard<std::mutex> lk(g_inject_mu);
  g_inject_name = entry ? entry : "*";
  g_inject_count.store(count < 0 ? 0 : count);
  return LB_OK;
}

size_t lb_quantize_workspace_bytes(void) { return kHeader; }

int lb_quantize_pack(int fmt, int group, const void *weight, int weight_dtype, int n, int k, uint8_t *codes,
                     uint16_t *scales, void *workspace, size_t workspace_bytes, void *stream) {
  if (injected("lb_quantize_pack")) return LB_ERR_INJECTED;
  if (!(fmt == LB_FMT_INT4 || fmt == LB_FMT_NF4 || fmt == LB_FMT_INT8) || n < 1 || k < 1 || group < 1 || group > k ||
      k % group || !weight || !codes || !scales || (weight_dtype != 0 && weight_dtype != 1))
    return LB_ERR_INVALID_ARGUMENT;
  if (!workspace || workspace_bytes < kHeader) return LB_ERR_WORKSPACE;
  const size_t wbytes = size_t(n) * k * (weight_dtype == 0 ? 4 : 2);
  const size_t cb = code_bytes(fmt, n, k), sb = size_t(n) * (k / group) * 2;
  if (overlaps(codes, cb, weight, wbytes) || overlaps(scales, sb, weight, wbytes) || overlaps(codes, cb, scales, sb) ||
      overlaps(workspace, kHeader, codes, cb) || overlaps(workspace, kHeader, scales, sb))
    return LB_ERR_ALIAS;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int *flags = static_cast<int *>(workspace);
  cudaError_t e = launch_quantize(fmt, group, weight, weight_dtype, n, k, codes, scales, flags, st);
  if (e != cudaSuccess) return cuda_status(e);
  int host_flags = 0;
  e = cudaMemcpyAsync(&host_flags, flags, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_status(e);
  if (host_flags & 1) return LB_ERR_NONFINITE;
  if (host_flags & 2) return LB_ERR_SCALE_OVERFLOW;
  return LB_OK;
}

int lb_dequantize(int fmt, int group, int n, int k, const uint8_t *codes, const uint16_t *scales, uint16_t *out,
                  void *stream) {
  if (injected("lb_dequantize")) return LB_ERR_INJECTED;
  if (!(fmt == LB_FMT_INT4 || fmt == LB_FMT_NF4 || fmt == LB_FMT_INT8) || n < 1 || k < 1 || group < 1 || group > k ||
      k % group || !codes || !scales || !out)
    return LB_ERR_INVALID_ARGUMENT;
  const size_t ob = size_t(n) * k * 2;
  if (overlaps(out, ob, codes, code_bytes(fmt, n, k)) || overlaps(out, ob, scales, size_t(n) * (k / group) * 2))
    return LB_ERR_ALIAS;
  return cuda_status(launch_dequantize(fmt, group, n, k, codes, scales, out, static_cast<cudaStream_t>(stream)));
}

int lb_linear_select(int fmt, int group, int m, int n, int k, int rank) {
  if (!valid_format(fmt) || m < 1 || n < 1 || k < 1) return LB_PATH_GENERIC;
  return select_path(fmt, fmt == LB_FMT_FP16 ? k : group, m, n, k, rank);
}

size_t lb_linear_workspace_bytes(int fmt, int group, int m, int n, int k, int rank) {
  if (!valid_format(fmt) || m < 1 || n < 1 || k < 1) return kHeader;
  const int g = fmt == LB_FMT_FP16 ? k : group;
  size_t best = 0;
  for (int path = LB_PATH_GEMV; path <= LB_PATH_GENERIC; ++path) {
    const size_t b = linear_ws(path, fmt, g, m, n, k, rank);
    if (b > best) best = b;
  }
  return best;
}

int lb_linear_path(int path, int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                   const uint16_t *scales, const uint16_t *down, const uint16_t *up, int rank, const uint16_t *bias,
                   uint16_t *y, void *workspace, size_t workspace_bytes, void *stream) {
  if (injected("lb_linear")) return LB_ERR_INJECTED;
  int s = validate_linear(fmt, group, m, n, k, x, codes, scales, down, up, rank, y);
  if (s != LB_OK) return s;
  if (!down) rank = 0;
  if (fmt == LB_FMT_FP16) group = k;
  const int auto_path = select_path(fmt, group, m, n, k, rank);
  if (path == LB_PATH_AUTO) path = auto_path;
  // a requested fast path must fit the problem and the pointers
  const bool fast_ptrs = aligned16(x) && aligned16(codes) && aligned16(y) && aligned16(workspace) &&
                         (!down || (aligned16(down) && aligned16(up)));
  if (path == LB_PATH_GEMV && (!gemv_supported(fmt, group, m, n, k) || !fast_ptrs)) {
    if (auto_path == LB_PATH_GEMV) path = LB_PATH_GENERIC; else return LB_ERR_UNSUPPORTED;
  }
  if (path == LB_PATH_TC && (!tc_supported(fmt, group, m, n, k, rank) || !fast_ptrs)) {
    if (auto_path == LB_PATH_TC) path = LB_PATH_GENERIC; else return LB_ERR_UNSUPPORTED;
  }
  if (path != LB_PATH_GEMV && path != LB_PATH_TC && path != LB_PATH_GENERIC) return LB_ERR_INVALID_ARGUMENT;
  const size_t need = linear_ws(path, fmt, group, m, n, k, rank);
  if (!workspace || workspace_bytes < need) return LB_ERR_WORKSPACE;
  if (linear_alias_status(fmt, group, m, n, k, x, codes, scales, down, up, rank, bias, y) != LB_OK ||
      overlaps(y, size_t(m) * n * 2, workspace, need))
    return LB_ERR_ALIAS;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  int *err = reinterpret_cast<int *>(ws);
  uint16_t *z = rank > 0 ? reinterpret_cast<uint16_t *>(ws + kHeader) : nullptr;
  uint8_t *rest = ws + kHeader + z_bytes(m, rank);
  cudaError_t e = cudaSuccess;
  if (z && path == LB_PATH_GEMV) {   // the projection inside the GEMV launch when it qualifies
    bool fused = false;
    e = launch_gemv_fused_z(fmt, group, m, n, k, x, codes, scales, down, up, rank, bias, y, rest,
                            reinterpret_cast<int *>(ws + kCounterOffset), reinterpret_cast<float *>(z), err, st, &fused);
    if (e != cudaSuccess) return cuda_status(e);
    if (fused) return LB_OK;
  }
  if (z) {
    if (path == LB_PATH_TC && z_on_tc(m, k, rank)) {
      float *zpart = reinterpret_cast<float *>(rest + align256(tc_partial_bytes(m, n, k)));
      e = cudaMemsetAsync(z, 0, size_t(m) * 32 * 2, st);
      if (e == cudaSuccess)
        e = launch_tc(LB_FMT_FP16, k, m, rank, k, x, reinterpret_cast<const uint8_t *>(down), nullptr, nullptr,
                      nullptr, 0, nullptr, z, 32, zpart, reinterpret_cast<int *>(ws + kCounterOffset), err, st);
    } else {
      e = launch_lowrank_project(m, k, rank, 32, x, down, z, st);
    }
    if (e != cudaSuccess) return cuda_status(e);
  }
  switch (path) {
    case LB_PATH_GEMV:
      e = launch_gemv(fmt, group, m, n, k, x, codes, scales, z, 32, up, rank, bias, nullptr, y, rest,
                      reinterpret_cast<int *>(ws + kCounterOffset), st);
      break;
    case LB_PATH_TC:
      e = launch_tc(fmt, group, m, n, k, x, codes, scales, z, up, rank, bias, y, n, reinterpret_cast<float *>(rest),
                    reinterpret_cast<int *>(ws + kCounterOffset), err, st);
      break;
    default: e = launch_linear_generic(fmt, group, m, n, k, x, codes, scales, z, up, rank, bias, y, st); break;
  }
  return cuda_status(e);
}

int lb_linear(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes, const uint16_t *scales,
              const uint16_t *down, const uint16_t *up, int rank, const uint16_t *bias, uint16_t *y, void *workspace,
              size_t workspace_bytes, void *stream) {
  return lb_linear_path(LB_PATH_AUTO, fmt, group, m, n, k, x, codes, scales, down, up, rank, bias, y, workspace,
                        workspace_bytes, stream);
}

int lb_linear_stacked(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                      const uint16_t *scales, const uint16_t *down, const uint16_t *up, const uint16_t *z_in,
                      int rank, const uint16_t *bias, const uint16_t *residual, uint16_t *y, void *workspace,
                      size_t workspace_bytes, void *stream) {
  if (injected("lb_linear_stacked")) return LB_ERR_INJECTED;
  if (!valid_format(fmt) || m < 1 || n < 1 || k < 1 || !x || !codes || !y) return LB_ERR_INVALID_ARGUMENT;
  if (fmt != LB_FMT_FP16 && (!scales || group < 1 || group > k || k % group)) return LB_ERR_INVALID_ARGUMENT;
  if (z_in && (down || !up)) return LB_ERR_INVALID_ARGUMENT;   // a given z replaces the projection
  if (!z_in && (down == nullptr) != (up == nullptr)) return LB_ERR_INVALID_ARGUMENT;
  if (up && (rank < 1 || rank > 128 || rank > k)) return LB_ERR_INVALID_ARGUMENT;
  if (int64_t(m) * k > (int64_t(1) << 40) || int64_t(n) * k > (int64_t(1) << 40)) return LB_ERR_INVALID_ARGUMENT;
  if (!up) rank = 0;
  if (fmt == LB_FMT_FP16) group = k;
  if (!gemv_supported(fmt, group, m, n, k) || !aligned16(x) || !aligned16(codes) || !aligned16(y) ||
      !aligned16(workspace) || (down && !aligned16(down)) || (up && !aligned16(up)) || (z_in && !aligned16(z_in)))
    return LB_ERR_UNSUPPORTED;
  const size_t need = kHeader + z_bytes(m, rank) + align256(gemv_workspace_bytes(fmt, m, n, k));
  if (!workspace || workspace_bytes < need) return LB_ERR_WORKSPACE;
  const size_t yb = size_t(m) * n * 2;
  if (overlaps(y, yb, x, size_t(m) * k * 2) || overlaps(y, yb, codes, code_bytes(fmt, n, k)) ||
      (scales && overlaps(y, yb, scales, size_t(n) * (k / group) * 2)) ||
      (bias && overlaps(y, yb, bias, size_t(n) * 2)) || (down && overlaps(y, yb, down, size_t(rank) * k * 2)) ||
      (up && overlaps(y, yb, up, size_t(n) * rank * 2)) || (residual && overlaps(y, yb, residual, yb)) ||
      overlaps(y, yb, workspace, need))
    return LB_ERR_ALIAS;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  const int zs = (rank + 31) / 32 * 32;
  const uint16_t *z = z_in;
  cudaError_t e = cudaSuccess;
  if (rank > 0 && !z_in) {
    uint16_t *zw = reinterpret_cast<uint16_t *>(ws + kHeader);
    e = launch_lowrank_project(m, k, rank, zs, x, down, zw, st);
    z = zw;
  }
  if (e == cudaSuccess)
    e = launch_gemv(fmt, group, m, n, k, x, codes, scales, z, zs, up, rank, bias, residual, y,
                    ws + kHeader + z_bytes(m, rank), reinterpret_cast<int *>(ws + kCounterOffset), st);
  return cuda_status(e);
}

int lb_workspace_status(const void *workspace, void *stream) {
  if (!workspace) return LB_ERR_INVALID_ARGUMENT;
  int flag = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&flag, workspace, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_status(e);
  return flag;
}

int lb_workspace_check(void *workspace, size_t workspace_bytes, void *stream) {
  if (!workspace || workspace_bytes < kHeader) return LB_ERR_INVALID_ARGUMENT;
  const int flag = lb_workspace_status(workspace, stream);
  if (flag == LB_OK || flag == LB_ERR_CUDA) return flag;
  // a wait gave up: arrivals may have landed after the counters were reset, so the
  // status word and every counter start again from zero
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(workspace, 0, kHeader, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_status(e);
  return flag;
}

int lb_test_wait_override(long long wait_cycles, int missing_arrivals) {
  set_wait_override(wait_cycles, missing_arrivals);
  return LB_OK;
}

int lb_rmsnorm(const uint16_t *x, const uint16_t *residual, uint16_t *residual_out, const uint16_t *gamma,
               uint16_t *out, int rows, int dim, float eps, void *stream) {
  if (injected("lb_rmsnorm")) return LB_ERR_INJECTED;
  if (!x || !gamma || !out || rows < 1 || dim < 8 || dim % 8 || dim > 16384 || !(eps >= 0.f)) return LB_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || !aligned16(gamma) || !aligned16(out) || (residual && !aligned16(residual)) ||
      (residual_out && !aligned16(residual_out)))
    return LB_ERR_INVALID_ARGUMENT;
  const size_t b = size_t(rows) * dim * 2;
  if (overlaps(out, b, x, b) || (residual && overlaps(out, b, residual, b)) || (residual_out && overlaps(out, b, residual_out, b)))
    return LB_ERR_ALIAS;
  return cuda_status(launch_rmsnorm(x, residual, residual_out, gamma, out, rows, dim, eps, static_cast<cudaStream_t>(stream)));
}

int lb_rope(uint16_t *q, uint16_t *k, const int32_t *positions, const uint16_t *cos_table, const uint16_t *sin_table,
            int table_rows, int tokens, int heads, int kv_heads, int head_dim, int q_stride, int k_stride, void *stream) {
  if (injected("lb_rope")) return LB_ERR_INJECTED;
  if (!q || !k || !positions || !cos_table || !sin_table || table_rows < 1 || tokens < 1 || heads < 1 ||
      kv_heads < 1 || head_dim < 2 || head_dim % 2 || q_stride < heads * head_dim || k_stride < kv_heads * head_dim)
    return LB_ERR_INVALID_ARGUMENT;
  return cuda_status(launch_rope(q, k, positions, cos_table, sin_table, table_rows, tokens, heads, kv_heads, head_dim,
                                 q_stride, k_stride, static_cast<cudaStream_t>(stream)));
}

int lb_kv_append(const uint16_t *k, const uint16_t *v, int kv_stride, uint16_t *k_cache, uint16_t *v_cache,
                 const int32_t *lengths, int batch, int kv_heads, int head_dim, int max_pos, void *stream) {
  if (injected("lb_kv_append")) return LB_ERR_INJECTED;
  if (!k || !v || !k_cache || !v_cache || !lengths || batch < 1 || kv_heads < 1 || head_dim < 1 || max_pos < 1 ||
      kv_stride < kv_heads * head_dim)
    return LB_ERR_INVALID_ARGUMENT;
  return cuda_status(launch_kv_append(k, v, kv_stride, k_cache, v_cache, lengths, batch, kv_heads, head_dim, max_pos,
                                      static_cast<cudaStream_t>(stream)));
}

size_t lb_attention_workspace_bytes(int batch, int heads, int max_pos) {
  if (batch < 1 || heads < 1 || max_pos < 1) return kHeader;
  return kHeader + attention_scratch_bytes(batch, heads, 16);
}

namespace {
// Attention workspace: the linear workspace's arrival counters (the same header, so one
// buffer can serve both on a stream) and the position-split scratch after it.  A missing
// or short workspace only limits the splits.
void attention_ws(void *workspace, size_t workspace_bytes, int **counters, void **scratch, size_t *scratch_bytes) {
  *counters = nullptr;
  *scratch = nullptr;
  *scratch_bytes = 0;
  if (workspace && workspace_bytes > kHeader && aligned16(workspace)) {
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    *counters = reinterpret_cast<int *>(ws + kCounterOffset);
    *scratch = ws + kHeader;
    *scratch_bytes = workspace_bytes - kHeader;
  }
}

bool attention_shape_ok(int batch, int heads, int kv_heads, int head_dim, int max_pos) {
  return batch >= 1 && heads >= 1 && kv_heads >= 1 && heads % kv_heads == 0 && heads / kv_heads <= 8 &&
         head_dim == 64 && max_pos >= 1 && int64_t(batch) * kv_heads * max_pos <= (int64_t(1) << 31);
}
}  // namespace

int lb_attention_decode(const uint16_t *q, int q_stride, const uint16_t *k_cache, const uint16_t *v_cache,
                        const int32_t *lengths, uint16_t *out, int batch, int heads, int kv_heads, int head_dim,
                        int max_pos, float scale, void *workspace, size_t workspace_bytes, void *stream) {
  if (injected("lb_attention_decode")) return LB_ERR_INJECTED;
  if (!q || !k_cache || !v_cache || !lengths || !out || !attention_shape_ok(batch, heads, kv_heads, head_dim, max_pos) ||
      q_stride < heads * head_dim)
    return LB_ERR_INVALID_ARGUMENT;
  if (!aligned16(k_cache) || !aligned16(v_cache) || !aligned16(q) || q_stride % 8) return LB_ERR_INVALID_ARGUMENT;
  int *counters;
  void *scratch;
  size_t sb;
  attention_ws(workspace, workspace_bytes, &counters, &scratch, &sb);
  return cuda_status(launch_attention_decode(q, q_stride, k_cache, v_cache, lengths, out, batch, heads, kv_heads,
                                             head_dim, max_pos, scale, counters, scratch, sb,
                                             static_cast<cudaStream_t>(stream)));
}

int lb_attention_decode_rope(const uint16_t *q, int q_stride, const uint16_t *k_new, const uint16_t *v_new,
                             int kv_stride, const uint16_t *cos_table, const uint16_t *sin_table, int table_rows,
                             uint16_t *k_cache, uint16_t *v_cache, const int32_t *lengths, uint16_t *out, int batch,
                             int heads, int kv_heads, int head_dim, int max_pos, float scale, void *workspace,
                             size_t workspace_bytes, void *stream) {
  if (injected("lb_attention_decode_rope")) return LB_ERR_INJECTED;
  if (!q || !k_new || !v_new || !cos_table || !sin_table || !k_cache || !v_cache || !lengths || !out ||
      !attention_shape_ok(batch, heads, kv_heads, head_dim, max_pos) || table_rows < 1 ||
      q_stride < heads * head_dim || kv_stride < kv_heads * head_dim)
    return LB_ERR_INVALID_ARGUMENT;
  if (!aligned16(k_cache) || !aligned16(v_cache) || !aligned16(q) || q_stride % 8) return LB_ERR_INVALID_ARGUMENT;
  // strided row blocks: the last row ends width elements after its start
  const size_t ob = size_t(batch) * heads * head_dim * 2;
  const size_t qb = (size_t(batch - 1) * q_stride + size_t(heads) * head_dim) * 2;
  const size_t kb = (size_t(batch - 1) * kv_stride + size_t(kv_heads) * head_dim) * 2;
  if (overlaps(out, ob, q, qb) || overlaps(out, ob, k_new, kb) || overlaps(out, ob, v_new, kb) ||
      overlaps(out, ob, workspace, workspace_bytes))
    return LB_ERR_ALIAS;
  int *counters;
  void *scratch;
  size_t sb;
  attention_ws(workspace, workspace_bytes, &counters, &scratch, &sb);
  return cuda_status(launch_attention_decode_rope(q, q_stride, k_new, v_new, kv_stride, cos_table, sin_table,
                                                  table_rows, k_cache, v_cache, lengths, out, batch, heads, kv_heads,
                                                  head_dim, max_pos, scale, counters, scratch, sb,
                                                  static_cast<cudaStream_t>(stream)));
}

namespace {
int row_project(int mode, const uint16_t *x, const uint16_t *res, uint16_t *res_out, const uint16_t *gamma,
                uint16_t *out, int rows, int dim, int in_stride, float eps, const uint16_t *down, int rank, uint16_t *z,
                void *stream) {
  if (!x || !out || rows < 1 || dim < 8 || dim % 8 || dim > 16384) return LB_ERR_INVALID_ARGUMENT;
  if ((down == nullptr) != (z == nullptr) || (down && (rank < 1 || rank > 128))) return LB_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || !aligned16(out) || (res && !aligned16(res)) || (res_out && !aligned16(res_out)) ||
      (gamma && !aligned16(gamma)) || (down && (!aligned16(down) || !aligned16(z))))
    return LB_ERR_INVALID_ARGUMENT;
  return cuda_status(launch_row_project(mode, x, res, res_out, gamma, out, rows, dim, in_stride, eps, down, rank, z,
                                        static_cast<cudaStream_t>(stream)));
}
}  // namespace

int lb_rmsnorm_project(const uint16_t *x, const uint16_t *residual, uint16_t *residual_out, const uint16_t *gamma,
                       uint16_t *out, int rows, int dim, float eps, const uint16_t *down, int rank, uint16_t *z,
                       void *stream) {
  if (injected("lb_rmsnorm_project")) return LB_ERR_INJECTED;
  if (!gamma || !(eps >= 0.f)) return LB_ERR_INVALID_ARGUMENT;
  const size_t b = size_t(rows) * dim * 2;
  if (rows > 0 && dim > 0 && (overlaps(out, b, x, b) || (residual && overlaps(out, b, residual, b)) ||
                              (residual_out && overlaps(out, b, residual_out, b))))
    return LB_ERR_ALIAS;
  return row_project(0, x, residual, residual_out, gamma, out, rows, dim, dim, eps, down, rank, z, stream);
}

int lb_silu_mul_project(const uint16_t *gate, const uint16_t *up, int in_stride, uint16_t *out, int rows, int cols,
                        const uint16_t *down, int rank, uint16_t *z, void *stream) {
  if (injected("lb_silu_mul_project")) return LB_ERR_INJECTED;
  if (!up || in_stride < cols || in_stride % 8 || !aligned16(up)) return LB_ERR_INVALID_ARGUMENT;
  return row_project(1, gate, up, nullptr, nullptr, out, rows, cols, in_stride, 0.f, down, rank, z, stream);
}

int lb_silu_mul(const uint16_t *gate, const uint16_t *up, int in_stride, uint16_t *out, int rows, int cols,
                void *stream) {
  if (injected("lb_silu_mul")) return LB_ERR_INJECTED;
  if (!gate || !up || !out || rows < 1 || cols < 1 || in_stride < cols) return LB_ERR_INVALID_ARGUMENT;
  return cuda_status(launch_silu_mul(gate, up, in_stride, out, rows, cols, static_cast<cudaStream_t>(stream)));
}

int lb_add(const uint16_t *a, const uint16_t *b, uint16_t *out, int64_t count, void *stream) {
  if (injected("lb_add")) return LB_ERR_INJECTED;
  if (!a || !b || !out || count < 1) return LB_ERR_INVALID_ARGUMENT;
  return cuda_status(launch_add(a, b, out, count, static_cast<cudaStream_t>(stream)));
}

int lb_embed(const int64_t *ids, const uint16_t *table, uint16_t *out, int64_t tokens, int dim, int64_t vocab,
             void *stream) {
  if (injected("lb_embed")) return LB_ERR_INJECTED;
  if (!ids || !table || !out || tokens < 1 || dim < 1 || vocab < 1) return LB_ERR_INVALID_ARGUMENT;
  return cuda_status(launch_embed(ids, table, out, tokens, dim, vocab, static_cast<cudaStream_t>(stream)));
}

size_t lb_argmax_workspace_bytes(int, int) { return 0; }

int lb_argmax(const uint16_t *logits, int rows, int vocab, int64_t *out, void *, size_t, void *stream) {
  if (injected("lb_argmax")) return LB_ERR_INJECTED;
  if (!logits || !out || rows < 1 || vocab < 1) return LB_ERR_INVALID_ARGUMENT;
  return cuda_status(launch_argmax(logits, rows, vocab, out, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
