// Allocation-free decode GEMV: lb_linear_gemv_noalloc.
//
// Some callers of this library cannot hand it a workspace: a host application that
// links liblowbit through the C ABI with a device-memory budget owned by another
// allocator it may not call into, or code on a latency-critical thread where a first
// cudaMalloc would block and synchronise the device.  For them this entry point runs
// the decode GEMV (M <= 64) with its scratch -- the correction projection z, split-K
// fp32 partials and arrival counters -- in one fixed array compiled into the library,
// so a call allocates nothing.
//
// The array below lives in every GPU that loads the library until the process exits.
// Host code must not use its name as a device address (on the host it is only a
// stand-in symbol); the device address is looked up once per device with
// cudaGetSymbolAddress while that device is current, on the first call made there.
#include <mutex>

#include "common.cuh"

namespace lowbit_host {
bool gemv_supported(int fmt, int group, int m, int n, int k);
size_t gemv_workspace_bytes(int fmt, int m, int n, int k);
cudaError_t launch_lowrank_project(int m, int k, int rank, int zs, const uint16_t *x, const uint16_t *v, uint16_t *z,
                                   cudaStream_t st);
cudaError_t launch_gemv(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                        const uint16_t *scales, const uint16_t *z, int zs, const uint16_t *up, int rank,
                        const uint16_t *bias, const uint16_t *resid, uint16_t *y, void *scratch, int *counters,
                        cudaStream_t st);
cudaError_t launch_gemv_fused_z(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                                const uint16_t *scales, const uint16_t *down, const uint16_t *up, int rank,
                                const uint16_t *bias, uint16_t *y, void *scratch, int *counters, float *zpart,
                                int *err, cudaStream_t st, bool *fused);
size_t gemv_fused_zpart_bytes(int m);
}  // namespace lowbit_host

namespace {

// Layout: [0, 16 KiB) arrival counters (4096 ints) | [16 KiB, +256) status word (a fused
// projection's timed-out wait) | then 64 KiB of z (or the fused projection's fp32 slices) |
// rest: partials.
constexpr size_t kCounterBytes = 4096 * sizeof(int);
constexpr size_t kStatusOffset = kCounterBytes;
constexpr size_t kZOffset = kStatusOffset + 256;
constexpr size_t kZBytes = 64 << 10;
constexpr size_t kPartialOffset = kZOffset + kZBytes;

static __device__ __align__(256) unsigned char g_noalloc_scratch[LB_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void *g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device).
cudaError_t scratch_address(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (!g_scratch_addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return cudaSuccess;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int lb_linear_gemv_noalloc(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                                      const uint16_t *scales, const uint16_t *down, const uint16_t *up, int rank,
                                      const uint16_t *bias, uint16_t *y, void *stream) {
  using namespace lowbit_host;
  if (injected("lb_linear_gemv_noalloc")) return LB_ERR_INJECTED;
  if (!(fmt == LB_FMT_INT4 || fmt == LB_FMT_NF4 || fmt == LB_FMT_INT8 || fmt == LB_FMT_FP16) || m < 1 || n < 1 ||
      k < 1 || !x || !codes || !y || (fmt != LB_FMT_FP16 && (!scales || group < 1 || group > k || k % group)))
    return LB_ERR_INVALID_ARGUMENT;
  if ((down == nullptr) != (up == nullptr) || (down && (rank < 1 || rank > 32 || rank > n || rank > k)))
    return LB_ERR_INVALID_ARGUMENT;
  if (fmt == LB_FMT_FP16) group = k;
  if (!down) rank = 0;
  if (!gemv_supported(fmt, group, m, n, k) || !aligned16(x) || !aligned16(codes) || !aligned16(y) ||
      (down && (!aligned16(down) || !aligned16(up))))
    return LB_ERR_UNSUPPORTED;   // only the decode GEMV (M <= 64, aligned rows) has this variant
  if (size_t(m) * 32 * 2 > kZBytes || gemv_fused_zpart_bytes(m) > kZBytes ||
      gemv_workspace_bytes(fmt, m, n, k) > size_t(LB_NOALLOC_SCRATCH_BYTES) - kPartialOffset)
    return LB_ERR_WORKSPACE;     // the problem needs more scratch than the fixed array holds
  if (linear_alias_status(fmt, group, m, n, k, x, codes, scales, down, up, rank, bias, y) != LB_OK)
    return LB_ERR_ALIAS;
  void *base = nullptr;
  cudaError_t e = scratch_address(&base);
  if (e != cudaSuccess) return LB_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *s = static_cast<uint8_t *>(base);
  int *counters = reinterpret_cast<int *>(s);
  // The array keeps whatever the previous call left; the counters and the status word
  // (contiguous at its start) must start at zero.
  e = cudaMemsetAsync(counters, 0, kZOffset, st);
  if (e == cudaSuccess && rank > 0) {   // the same fused projection lb_linear would run
    bool fused = false;
    e = launch_gemv_fused_z(fmt, group, m, n, k, x, codes, scales, down, up, rank, bias, y, s + kPartialOffset,
                            counters, reinterpret_cast<float *>(s + kZOffset),
                            reinterpret_cast<int *>(s + kStatusOffset), st, &fused);
    if (e != cudaSuccess || fused) return e == cudaSuccess ? LB_OK : LB_ERR_CUDA;
  }
  uint16_t *z = nullptr;
  if (e == cudaSuccess && rank > 0) {
    z = reinterpret_cast<uint16_t *>(s + kZOffset);
    e = launch_lowrank_project(m, k, rank, 32, x, down, z, st);
  }
  if (e == cudaSuccess)
    e = launch_gemv(fmt, group, m, n, k, x, codes, scales, z, 32, up, rank, bias, nullptr, y, s + kPartialOffset,
                    counters, st);
  return e == cudaSuccess ? LB_OK : LB_ERR_CUDA;
}

// SYNCHRONOUS: waits for `stream`, then returns the status word of the current device's
// array (LB_OK, or LB_ERR_TIMEOUT when a bounded wait of the last call on it gave up, in
// which case its output is not valid) and clears it with the arrival counters.
extern "C" int lb_noalloc_status(void *stream) {
  void *base = nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = scratch_address(&base);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return LB_ERR_CUDA;
  uint8_t *s = static_cast<uint8_t *>(base);
  int flag = 0;
  e = cudaMemcpyAsync(&flag, s + kStatusOffset, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && flag != LB_OK) {
    e = cudaMemsetAsync(s, 0, kZOffset, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  return e == cudaSuccess ? flag : LB_ERR_CUDA;
}
