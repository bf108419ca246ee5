// Shared device helpers for the low-bit kernels (sm_100a only).
#pragma once
#include <mutex>
#include <unordered_map>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "lowbit.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "liblowbit is built for sm_100a (B200) only"
#endif

namespace lowbit {

// The 16-entry NF4 codebook of torch_npu_lowbit.py:17-20, fp32.
__host__ __device__ constexpr float nf4_value(int i) {
  constexpr float t[16] = {-1.f, -.6961928009986877f, -.5250730514526367f, -.39491748809814453f,
                           -.28444138169288635f, -.18477343022823334f, -.09105003625154495f, 0.f,
                           .07958029955625534f, .16093020141124725f, .24611230194568634f,
                           .33791524171829224f, .44070982933044434f, .5626170039176941f,
                           .7229568362236023f, 1.f};
  return t[i];
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Runtime-indexed copy of the codebook in constant memory (a runtime index into the
// constexpr table above would be lowered to a per-thread stack array).
static __constant__ float c_nf4[16] = {
    -1.f, -.6961928009986877f, -.5250730514526367f, -.39491748809814453f, -.28444138169288635f,
    -.18477343022823334f, -.09105003625154495f, 0.f, .07958029955625534f, .16093020141124725f,
    .24611230194568634f, .33791524171829224f, .44070982933044434f, .5626170039176941f, .7229568362236023f, 1.f};

// Fill the per-lane-replicated byte->half2 NF4 table used by the decode and GEMM
// kernels: word (e * STRIDE + l) = (NF4h[e & 15], NF4h[e >> 4]) for every lane l < 32
// (STRIDE = 32 packs the entries; 64 leaves a 128-byte gap so that one byte_perm forms
// the address).  Each thread writes whole entries with 16-byte stores rotated by lane,
// so the stores of a warp hit distinct bank groups.
template <int STRIDE = 32>
__device__ __forceinline__ void fill_nf4_pair_lut(uint32_t *lut) {
  const int lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < 256; e += blockDim.x) {
    const __half2 v = __halves2half2(__float2half_rn(c_nf4[e & 15]), __float2half_rn(c_nf4[e >> 4]));
    const uint32_t u = h2_as_u32(v);
    const uint4 q = make_uint4(u, u, u, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) reinterpret_cast<uint4 *>(lut + e * STRIDE)[(j + lane) & 7] = q;
  }
}

// acc += a.lo * b.lo + a.hi * b.hi with exact fp16 products, fp32 accumulation
// (mixed-precision fma of PTX ISA 8.6, one instruction per product).
__device__ __forceinline__ void fma2_f16_f32(float &acc, uint32_t a, uint32_t b) {
  asm("{\n\t.reg .f16 al, ah, bl, bh;\n\t"
      "mov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
      "fma.rn.f32.f16 %0, al, bl, %0;\n\tfma.rn.f32.f16 %0, ah, bh, %0;\n\t}"
      : "+f"(acc)
      : "r"(a), "r"(b));
}

// ---- 4-bit signed (two's complement nibble) -> fp16 pairs without conversions ----------
// For a 32-bit word holding 8 codes (element e in bits 4e..4e+3), produce half2 pairs
// p0 = (e0, e4), p1 = (e1, e5), p2 = (e2, e6), p3 = (e3, e7) holding the exact signed
// values ((c ^ 8) - 8).  The codes are OR-ed under the fp16 exponent of 1024 (0x6400)
// with bit 3 flipped, so the half equals 1024 + (c ^ 8) (or 1024 + 16 (c ^ 8) for the
// high nibble of each byte) and one exact fp16 subtract / fma recovers the value.
__device__ __forceinline__ uint32_t lop3_sel(uint32_t w, uint32_t mask, uint32_t bits) {
  // f = mask ? (w ^ bits) : bits; truth table over (a=w:0xF0, b=mask:0xCC, c=bits:0xAA)
  // = (0xCC & (0xF0 ^ 0xAA)) | (~0xCC & 0xAA) = 0x48 | 0x22 = 0x6A.
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(w), "r"(mask), "r"(bits));
  return r;
}

__device__ __forceinline__ void int4_word_to_h2(uint32_t w, uint32_t out[4]) {
  const uint32_t lo_mask = 0x000F000Fu, hi_mask = 0x00F000F0u;
  const uint32_t lo_bits = 0x64086408u, hi_bits = 0x64806480u;
  const __half2 lo_sub = __float2half2_rn(1032.f);                 // 1024 + 8
  const __half2 hi_mul = __float2half2_rn(0.0625f), hi_add = __float2half2_rn(-72.f);
  uint32_t a = lop3_sel(w, lo_mask, lo_bits);
  uint32_t b = lop3_sel(w, hi_mask, hi_bits);
  uint32_t w8 = w >> 8;
  uint32_t c = lop3_sel(w8, lo_mask, lo_bits);
  uint32_t d = lop3_sel(w8, hi_mask, hi_bits);
  out[0] = h2_as_u32(__hsub2(u32_as_h2(a), lo_sub));
  out[1] = h2_as_u32(__hfma2(u32_as_h2(b), hi_mul, hi_add));
  out[2] = h2_as_u32(__hsub2(u32_as_h2(c), lo_sub));
  out[3] = h2_as_u32(__hfma2(u32_as_h2(d), hi_mul, hi_add));
}

// ---- int8 -> fp16 pairs: bytes (b0,b1,b2,b3) -> (b0,b2), (b1,b3) exact -----------------
__device__ __forceinline__ void int8_word_to_h2(uint32_t w, uint32_t out[2]) {
  const uint32_t flipped = w ^ 0x80808080u;                        // u = b + 128
  const __half2 sub = __float2half2_rn(1152.f);                    // 1024 + 128
  uint32_t a = __byte_perm(flipped, 0x64646464u, 0x4240);          // (0x64:u0, 0x64:u2)
  uint32_t b = __byte_perm(flipped, 0x64646464u, 0x4341);          // (0x64:u1, 0x64:u3)
  out[0] = h2_as_u32(__hsub2(u32_as_h2(a), sub));
  out[1] = h2_as_u32(__hsub2(u32_as_h2(b), sub));
}

// ---- PDL (programmatic dependent launch) -------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

__device__ __forceinline__ uint4 ldg_nc_v4(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---- mbarriers (bounded waits) and bulk copies --------------------------------------
constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at 1.9 GHz

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t a, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t a) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait.  Returns false if the CTA aborted or the wait timed out.
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity, volatile int *abort_flag) {
  if (mbar_try_wait(a, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(a, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) { *abort_flag = 1; return false; }
  }
  return true;
}

// Time-bounded wait that ignores the abort flag (used to drain copies in flight).
__device__ __forceinline__ bool mbar_wait_drain(uint32_t a, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(a, parity))
    if (clock64() - t0 > kWaitCycles) return false;
  return true;
}


__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace lowbit

// Host-side launch helpers.
namespace lowbit_host {
// abi.cu: host-side fault injection, pointer-range overlap and the alias checks of a
// linear call (an output overlapping an input), shared by every linear entry point
bool injected(const char *entry);
bool overlaps(const void *a, size_t na, const void *b, size_t nb);
size_t code_bytes(int fmt, int64_t n, int64_t k);
int linear_alias_status(int fmt, int group, int m, int n, int k, const void *x, const void *codes, const void *scales,
                        const void *down, const void *up, int rank, const void *bias, const void *y);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) is a driver round trip: issue it once
// per (kernel, device) and whenever a larger size is requested.
inline cudaError_t ensure_dyn_smem(const void *func, int bytes) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, int> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t key = (uint64_t(reinterpret_cast<uintptr_t>(func)) << 6) ^ uint64_t(dev);
  std::lock_guard<std::mutex> lk(mu);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done[key] = bytes;
  return e;
}
bool pdl_enabled();  // defined in abi.cu (env LOWBIT_PDL, default on)

// cudaLaunchKernelEx with programmatic dependent launch when enabled: every kernel of
// this library calls griddepcontrol.wait before touching data a predecessor may write.
template <typename Kern, typename... Args>
inline cudaError_t launch_k(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}
}  // namespace lowbit_host
