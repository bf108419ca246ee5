// K1: quantize + pack (quantize_weight, torch_npu_lowbit.py:78-105) and the fp16
// dequantization of PackedWeight.dequantize (torch_npu_lowbit.py:67-75), bit-exact.
//
// Exactness notes: the reference computes in numpy fp32 with IEEE division and
// round-half-even; here every division is __fdiv_rn, rounding is rintf (half-even),
// fp32->fp16 is __float2half_rn, and the NF4 midpoints are formed with __fadd_rn so
// no contraction can change them.  Build without --use_fast_math.
#include "common.cuh"

namespace lowbit {

__device__ __forceinline__ float load_weight(const void *w, int dtype, int64_t i) {
  return dtype == 0 ? __ldg(reinterpret_cast<const float *>(w) + i)
                    : __half2float(__ldg(reinterpret_cast<const __half *>(w) + i));
}

__device__ __forceinline__ float format_limit(int fmt) {
  return fmt == LB_FMT_INT4 ? 7.f : (fmt == LB_FMT_NF4 ? 1.f : 127.f);
}

// Phase 1: one warp per group -> fp16 scale.  flags bit0: non-finite, bit1: overflow.
__global__ void quantize_scales_kernel(int fmt, const void *__restrict__ w, int dtype, int64_t groups,
                                       int group, __half *__restrict__ scales, int *__restrict__ flags) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t gi = warp; gi < groups; gi += nwarps) {
    const int64_t base = gi * group;
    float amax = 0.f;
    bool finite = true;
    for (int i = lane; i < group; i += 32) {
      const float v = load_weight(w, dtype, base + i);
      finite &= isfinite(v);
      amax = fmaxf(amax, fabsf(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    finite = __all_sync(0xffffffffu, finite);
    if (lane == 0) {
      if (!finite) atomicOr(flags, 1);
      const float s = __fdiv_rn(amax, format_limit(fmt));            // maximum / limit
      if (s > 65504.f) atomicOr(flags, 2);                             // > finfo(fp16).max
      scales[gi] = __float2half_rn(fmaxf(s, 5.9604644775390625e-08f)); // max(s, 2^-24) -> fp16
    }
  }
}

__device__ __forceinline__ uint32_t quantize_one(int fmt, float v, float sf) {
  const float x = __fdiv_rn(v, sf);                                    // values / scale
  if (fmt == LB_FMT_NF4) {
    // searchsorted(midpoints, x, side='left') == number of midpoints strictly below x
    uint32_t code = 0;
#pragma unroll
    for (int i = 0; i < 15; ++i) {
      const float mid = __fmul_rn(__fadd_rn(nf4_value(i), nf4_value(i + 1)), 0.5f);
      code += (mid < x) ? 1u : 0u;
    }
    return code;
  }
  const float lim = format_limit(fmt);
  const float r = fminf(fmaxf(rintf(x), -lim), lim);
  return uint32_t(int32_t(r)) & (fmt == LB_FMT_INT8 ? 0xFFu : 0xFu);
}

// Phase 2: codes.  4-bit: one thread per output byte (flat elements 2t, 2t+1, the even
// element in the low nibble, a zero high nibble past the end).  int8: one per byte.
__global__ void quantize_codes_kernel(int fmt, const void *__restrict__ w, int dtype, int64_t count,
                                      int group, const __half *__restrict__ scales,
                                      uint8_t *__restrict__ codes) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  if (fmt == LB_FMT_INT8) {
    for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < count; e += stride) {
      const float sf = __half2float(scales[e / group]);
      codes[e] = uint8_t(quantize_one(fmt, load_weight(w, dtype, e), sf));
    }
    return;
  }
  const int64_t nbytes = (count + 1) / 2;
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < nbytes; t += stride) {
    const int64_t e0 = 2 * t, e1 = 2 * t + 1;
    uint32_t lo = quantize_one(fmt, load_weight(w, dtype, e0), __half2float(scales[e0 / group]));
    uint32_t hi = 0;
    if (e1 < count) hi = quantize_one(fmt, load_weight(w, dtype, e1), __half2float(scales[e1 / group]));
    codes[t] = uint8_t(lo | (hi << 4));
  }
}

__device__ __forceinline__ __half code_value(int fmt, const uint8_t *codes, int64_t e) {
  if (fmt == LB_FMT_INT8) return __int2half_rn(int(int8_t(codes[e])));
  const uint32_t b = codes[e >> 1];
  const uint32_t c = (e & 1) ? (b >> 4) : (b & 15u);
  if (fmt == LB_FMT_INT4) return __int2half_rn(int((c ^ 8u)) - 8);
  return __float2half_rn(c_nf4[c]);
}

__global__ void dequantize_kernel(int fmt, const uint8_t *__restrict__ codes, const __half *__restrict__ scales,
                                  int64_t count, int group, __half *__restrict__ out) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < count; e += stride)
    out[e] = __hmul(code_value(fmt, codes, e), scales[e / group]);  // rn16(value * scale)
}

}  // namespace lowbit

namespace lowbit_host {

static int grid_for(int64_t work, int block) {
  int64_t g = (work + block - 1) / block;
  if (g > 148 * 32) g = 148 * 32;
  return int(g < 1 ? 1 : g);
}

cudaError_t launch_quantize(int fmt, int group, const void *w, int dtype, int n, int k, uint8_t *codes,
                            uint16_t *scales, int *flags, cudaStream_t stream) {
  const int64_t count = int64_t(n) * k, groups = count / group;
  cudaError_t e = cudaMemsetAsync(flags, 0, sizeof(int), stream);
  if (e != cudaSuccess) return e;
  lowbit::quantize_scales_kernel<<<grid_for(groups * 32, 256), 256, 0, stream>>>(
      fmt, w, dtype, groups, group, reinterpret_cast<__half *>(scales), flags);
  const int64_t work = fmt == LB_FMT_INT8 ? count : (count + 1) / 2;
  lowbit::quantize_codes_kernel<<<grid_for(work, 256), 256, 0, stream>>>(
      fmt, w, dtype, count, group, reinterpret_cast<const __half *>(scales), codes);
  return cudaGetLastError();
}

cudaError_t launch_dequantize(int fmt, int group, int n, int k, const uint8_t *codes, const uint16_t *scales,
                              uint16_t *out, cudaStream_t stream) {
  const int64_t count = int64_t(n) * k;
  lowbit::dequantize_kernel<<<grid_for(count, 256), 256, 0, stream>>>(
      fmt, codes, reinterpret_cast<const __half *>(scales), count, group, reinterpret_cast<__half *>(out));
  return cudaGetLastError();
}

}  // namespace lowbit_host
