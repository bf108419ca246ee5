// K2: decode dequant-GEMV for small M (x rows held in registers), with the rank-r
// correction applied in the epilogue.  HBM-bound by design:
//  * each lane streams 16-byte packed chunks of a weight row (128-bit coalesced loads,
//    L1 no-allocate), a warp covers up to 32 chunks of one row = one "K slice";
//  * the lane's slice of x (M rows) is loaded once and reused for every weight row;
//  * INT4 codes are unpacked in registers with lop3 + one exact fp16 op per pair,
//    NF4 codes through a per-lane-replicated 256-entry (byte -> half2) table in shared
//    memory (conflict-free), INT8 with byte_perm + one exact fp16 subtract;
//  * 4-bit weights are dequantized exactly as the reference does, rn16(code * scale),
//    and multiplied with x in fp32 (mixed-precision fma, exact products);
//  * partial sums are reduced with warp shuffles and across K slices in shared memory;
//  * epilogue: y = half(half(acc) [+ bias]) then half(y + half(z . U[n]^T)).
// Reference semantics: torch_npu_lowbit.py:67-75 (dequant), torch_npu_smollm.py:150-164.
#include "common.cuh"

namespace lowbit {

struct GemvParams {
  int m, n, k, group;
  const __half *x;       // [m, k]
  const uint8_t *codes;  // packed rows
  const __half *scales;  // [n, k/group] (unused for FP16)
  const __half *z;       // [m, 32] correction projection half(x . V^T), or null
  const __half *up;      // [n, rank]
  int rank;
  const __half *bias;    // [n] or null
  __half *y;             // [m, n]
  int nslices;           // K slices
  int slice_width;       // chunks per slice (<= 32)
  int warps_k;           // warps along K in a CTA (<= nslices)
  int rows_per_warp;     // rows handled by each warp (multiple of the unroll)
  int row_groups;        // warps along N in a CTA
  int prefetch;          // issue an L2 bulk prefetch of the CTA's weight slab first
};

template <int FMT> struct FmtTraits;
template <> struct FmtTraits<LB_FMT_INT4> { static constexpr int E = 32; static constexpr int BITS = 4; };
template <> struct FmtTraits<LB_FMT_NF4> { static constexpr int E = 32; static constexpr int BITS = 4; };
template <> struct FmtTraits<LB_FMT_INT8> { static constexpr int E = 16; static constexpr int BITS = 8; };
template <> struct FmtTraits<LB_FMT_FP16> { static constexpr int E = 8; static constexpr int BITS = 16; };

constexpr int kMaxWarps = 8;
constexpr int kMaxRowsCta = 64;
constexpr int kLutWords = 256 * 32;

template <int MT> struct Unroll { static constexpr int U = MT == 1 ? 8 : 4; };

// x pairs held by one lane for one activation row: 16 half2 (4-bit), 8 (int8), 4 (fp16)
template <int FMT> struct XRegs { static constexpr int N = FmtTraits<FMT>::E / 2; };

// Dot-product formulation (compile-time): 0 = mixed-precision fma (f16 x f16 -> f32),
// 1 = convert to fp32 + fmaf, 2 = fp16x2 fma into a per-chunk half2 partial,
// 3 = convert to fp32 + packed fp32x2 fma.  x pairs are stored in the matching type.
#ifndef LOWBIT_GEMV_DOT
#define LOWBIT_GEMV_DOT 3
#endif
constexpr int kDot = LOWBIT_GEMV_DOT;
constexpr bool kXFloat = kDot == 1 || kDot == 3;
struct XPair { uint32_t h; float2 f; };

__device__ __forceinline__ XPair make_xpair(uint32_t h2) {
  XPair x;
  if constexpr (kXFloat) x.f = __half22float2(u32_as_h2(h2)); else x.h = h2;
  return x;
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long A = (unsigned long long)__float_as_uint(a.x) | ((unsigned long long)__float_as_uint(a.y) << 32);
  unsigned long long B = (unsigned long long)__float_as_uint(b.x) | ((unsigned long long)__float_as_uint(b.y) << 32);
  unsigned long long C = (unsigned long long)__float_as_uint(c.x) | ((unsigned long long)__float_as_uint(c.y) << 32);
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(C) : "l"(A), "l"(B));
  return make_float2(__uint_as_float(uint32_t(C)), __uint_as_float(uint32_t(C >> 32)));
}

// per-chunk partial sum of 2 * pairs products
struct Part {
  float f; __half2 h; float2 f2;
  __device__ __forceinline__ void init() {
    if constexpr (kDot == 2) h = __float2half2_rn(0.f);
    else if constexpr (kDot == 3) f2 = make_float2(0.f, 0.f);
    else f = 0.f;
  }
  __device__ __forceinline__ void fma(uint32_t w2, const XPair &x) {
    if constexpr (kDot == 0) {
      fma2_f16_f32(f, w2, x.h);
    } else if constexpr (kDot == 1) {
      const float2 wf = __half22float2(u32_as_h2(w2));
      f = fmaf(wf.x, x.f.x, f);
      f = fmaf(wf.y, x.f.y, f);
    } else if constexpr (kDot == 2) {
      h = __hfma2(u32_as_h2(w2), u32_as_h2(x.h), h);
    } else {
      f2 = ffma2(__half22float2(u32_as_h2(w2)), x.f, f2);
    }
  }
  __device__ __forceinline__ float sum() const {
    if constexpr (kDot == 2) return __low2float(h) + __high2float(h);
    else if constexpr (kDot == 3) return f2.x + f2.y;
    else return f;
  }
};

template <int FMT>
__device__ __forceinline__ void load_x_chunk(const __half *xrow, int chunk, bool valid, XPair (&xr)[XRegs<FMT>::N]) {
  constexpr int E = FmtTraits<FMT>::E;
  constexpr int V = E / 8;  // uint4 loads
  uint32_t nat[E / 2];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    uint4 q = valid ? *reinterpret_cast<const uint4 *>(xrow + size_t(chunk) * E + v * 8) : make_uint4(0, 0, 0, 0);
    nat[v * 4 + 0] = q.x; nat[v * 4 + 1] = q.y; nat[v * 4 + 2] = q.z; nat[v * 4 + 3] = q.w;
  }
  if constexpr (FMT == LB_FMT_INT4) {
    // pairs (x0,x4),(x1,x5),(x2,x6),(x3,x7) per group of 8, matching int4_word_to_h2
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t A = nat[w * 4 + 0], B = nat[w * 4 + 1], C = nat[w * 4 + 2], D = nat[w * 4 + 3];
      xr[w * 4 + 0] = make_xpair(__byte_perm(A, C, 0x5410));
      xr[w * 4 + 1] = make_xpair(__byte_perm(A, C, 0x7632));
      xr[w * 4 + 2] = make_xpair(__byte_perm(B, D, 0x5410));
      xr[w * 4 + 3] = make_xpair(__byte_perm(B, D, 0x7632));
    }
  } else if constexpr (FMT == LB_FMT_INT8) {
    // pairs (x0,x2),(x1,x3) per group of 4, matching int8_word_to_h2
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t A = nat[w * 2 + 0], B = nat[w * 2 + 1];
      xr[w * 2 + 0] = make_xpair(__byte_perm(A, B, 0x5410));
      xr[w * 2 + 1] = make_xpair(__byte_perm(A, B, 0x7632));
    }
  } else {
#pragma unroll
    for (int i = 0; i < E / 2; ++i) xr[i] = make_xpair(nat[i]);
  }
}

// dot of one 16-byte weight chunk with the lane's x pairs for MT activation rows
template <int FMT, int MT, bool EXACT>
__device__ __forceinline__ void chunk_dot(const uint4 &q, __half2 s2, const uint32_t *lut_lane,
                                          const XPair (&xr)[MT][XRegs<FMT>::N], float (&acc)[MT]) {
  const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
  Part part[MT];
#pragma unroll
  for (int mm = 0; mm < MT; ++mm) part[mm].init();
  if constexpr (FMT == LB_FMT_INT4 || FMT == LB_FMT_NF4) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t p[4];
      if constexpr (FMT == LB_FMT_INT4) {
        int4_word_to_h2(wv[w], p);
      } else {
        const uint32_t b = wv[w];
        p[0] = lut_lane[((b << 5) & 0x1FE0u)];        // byte0 * 32 words
        p[1] = lut_lane[((b >> 3) & 0x1FE0u)];        // byte1
        p[2] = lut_lane[((b >> 11) & 0x1FE0u)];       // byte2
        p[3] = lut_lane[((b >> 19) & 0x1FE0u)];       // byte3
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (EXACT) p[j] = h2_as_u32(__hmul2(u32_as_h2(p[j]), s2));  // rn16(code * scale)
#pragma unroll
        for (int mm = 0; mm < MT; ++mm) part[mm].fma(p[j], xr[mm][w * 4 + j]);
      }
    }
    if constexpr (EXACT) {
#pragma unroll
      for (int mm = 0; mm < MT; ++mm) acc[mm] += part[mm].sum();
    } else {
      const float s = __low2float(s2);
#pragma unroll
      for (int mm = 0; mm < MT; ++mm) acc[mm] = fmaf(part[mm].sum(), s, acc[mm]);
    }
  } else if constexpr (FMT == LB_FMT_INT8) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t p[2];
      int8_word_to_h2(wv[w], p);
#pragma unroll
      for (int mm = 0; mm < MT; ++mm) {
        part[mm].fma(p[0], xr[mm][w * 2 + 0]);
        part[mm].fma(p[1], xr[mm][w * 2 + 1]);
      }
    }
    const float s = __low2float(s2);  // codes are exact; the group scale factors out
#pragma unroll
    for (int mm = 0; mm < MT; ++mm) acc[mm] = fmaf(part[mm].sum(), s, acc[mm]);
  } else {
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
      for (int mm = 0; mm < MT; ++mm) part[mm].fma(wv[w], xr[mm][w]);
#pragma unroll
    for (int mm = 0; mm < MT; ++mm) acc[mm] += part[mm].sum();
  }
}

template <int FMT, int MT, bool EXACT>
__global__ void __launch_bounds__(256) gemv_kernel(const GemvParams p) {
  constexpr int E = FmtTraits<FMT>::E;
  constexpr int U = Unroll<MT>::U;
  constexpr int XN = XRegs<FMT>::N;
  extern __shared__ __align__(16) uint32_t smem[];
  float *red = reinterpret_cast<float *>(smem);  // [warps_k][rows_cta][MT]
  uint32_t *lut = smem + kMaxWarps * kMaxRowsCta * 4;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wk = warp % p.warps_k, rg = warp / p.warps_k;
  const int rows_cta = p.row_groups * p.rows_per_warp;
  const int row_cta0 = blockIdx.x * rows_cta;
  const int64_t row_bytes = int64_t(p.k) * FmtTraits<FMT>::BITS / 8;
  const int chunks = p.k / E;

  pdl_launch();
  if (p.prefetch && threadIdx.x == 0) {
    // weights are read-only for the whole program, so they may be requested before
    // the predecessor kernel finishes
    const int rows = min(rows_cta, p.n - row_cta0);
    const uint8_t *base = p.codes + int64_t(row_cta0) * row_bytes;
    int64_t total = int64_t(rows) * row_bytes;
    for (int64_t off = 0; off < total; off += 65536)
      prefetch_l2_bulk(base + off, uint32_t(total - off < 65536 ? total - off : 65536));
  }
  if constexpr (FMT == LB_FMT_NF4) {
    fill_nf4_pair_lut(lut);
    __syncthreads();
  }
  pdl_wait();

  float acc[16][MT];  // rows_per_warp <= 16
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int mm = 0; mm < MT; ++mm) acc[i][mm] = 0.f;

  const int groups_per_row = p.k / p.group;
  const uint32_t *lut_lane = lut + lane;
  const int row_w0 = row_cta0 + rg * p.rows_per_warp;

  for (int s = wk; s < p.nslices; s += p.warps_k) {
    const int chunk = s * p.slice_width + lane;
    const bool active = lane < p.slice_width && chunk < chunks;
    XPair xr[MT][XN];
#pragma unroll
    for (int mm = 0; mm < MT; ++mm) load_x_chunk<FMT>(p.x + size_t(mm) * p.k, chunk, active && mm < p.m, xr[mm]);
    const int gidx = active ? (chunk * E) / p.group : 0;
#pragma unroll
    for (int i0 = 0; i0 < 16; i0 += U) {
      if (i0 >= p.rows_per_warp) break;
      uint4 q[U];
      __half2 s2[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int row = row_w0 + i0 + u;
        const bool ok = active && row < p.n;
        q[u] = ok ? ldg_nc_v4(p.codes + int64_t(row) * row_bytes + int64_t(chunk) * 16) : make_uint4(0, 0, 0, 0);
        if constexpr (FMT != LB_FMT_FP16) {
          const __half sc = ok ? p.scales[int64_t(row) * groups_per_row + gidx] : __float2half(0.f);
          s2[u] = __halves2half2(sc, sc);
        } else {
          s2[u] = __float2half2_rn(1.f);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) chunk_dot<FMT, MT, EXACT>(q[u], s2[u], lut_lane, xr, acc[i0 + u]);
    }
  }

  // reduce across lanes, then across K slices through shared memory
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (i >= p.rows_per_warp) break;
#pragma unroll
    for (int mm = 0; mm < MT; ++mm) {
      const float v = warp_sum(acc[i][mm]);
      if (lane == 0) red[(wk * rows_cta + rg * p.rows_per_warp + i) * MT + mm] = v;
    }
  }
  __syncthreads();

  for (int idx = threadIdx.x; idx < rows_cta * p.m; idx += blockDim.x) {
    const int mm = idx / rows_cta, rl = idx % rows_cta;
    const int n = row_cta0 + rl;
    if (n >= p.n || mm >= MT) continue;
    float v = 0.f;
    for (int w = 0; w < p.warps_k; ++w) v += red[(w * rows_cta + rl) * MT + mm];
    __half yq = __float2half_rn(v);
    if (p.bias) yq = __float2half_rn(__half2float(yq) + __half2float(p.bias[n]));
    if (p.z) {
      const __half *zr = p.z + mm * 32;
      const __half *ur = p.up + int64_t(n) * p.rank;
      float d = 0.f;
      for (int r = 0; r < p.rank; ++r) d = fmaf(__half2float(zr[r]), __half2float(ur[r]), d);
      yq = __float2half_rn(__half2float(yq) + __half2float(__float2half_rn(d)));
    }
    p.y[int64_t(mm) * p.n + n] = yq;
  }
}

// z[m, r] = half(sum_k x[m,k] V[r,k]) for r < rank (zero for rank <= r < 32):
// one CTA per (r, m-tile of up to 8 rows); 8 warps split K, 16-byte loads of V and x.
__global__ void __launch_bounds__(256) lowrank_project_kernel(int m, int k, int rank, const __half *__restrict__ x,
                                                              const __half *__restrict__ v, __half *__restrict__ z) {
  __shared__ float red[8][8];
  const int r = blockIdx.x, m0 = blockIdx.y * 8;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  pdl_launch();
  pdl_wait();
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  if (r < rank) {
    const __half *vr = v + int64_t(r) * k;
    for (int c = threadIdx.x; c < k / 8; c += blockDim.x) {
      const uint4 w = *reinterpret_cast<const uint4 *>(vr + c * 8);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (m0 + i < m) {
          const uint4 xv = *reinterpret_cast<const uint4 *>(x + int64_t(m0 + i) * k + c * 8);
          fma2_f16_f32(acc[i], w.x, xv.x);
          fma2_f16_f32(acc[i], w.y, xv.y);
          fma2_f16_f32(acc[i], w.z, xv.z);
          fma2_f16_f32(acc[i], w.w, xv.w);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float s = warp_sum(acc[i]);
    if (lane == 0) red[warp][i] = s;
  }
  __syncthreads();
  if (threadIdx.x < 8 && m0 + threadIdx.x < m) {
    float s = 0.f;
    for (int w = 0; w < 8; ++w) s += red[w][threadIdx.x];
    z[int64_t(m0 + threadIdx.x) * 32 + r] = __float2half_rn(r < rank ? s : 0.f);
  }
}

// Shape-general fallback (any K, any group, odd element counts): one warp per output
// (m, n), elements decoded one at a time.  Same staging as the fast paths.
__global__ void linear_generic_kernel(int fmt, int m, int n, int k, int group, const __half *__restrict__ x,
                                      const uint8_t *__restrict__ codes, const __half *__restrict__ scales,
                                      const __half *__restrict__ z, const __half *__restrict__ up, int rank,
                                      const __half *__restrict__ bias, __half *__restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  pdl_launch();
  pdl_wait();
  if (warp >= int64_t(m) * n) return;
  const int mm = int(warp / n), nn = int(warp % n);
  const bool per_row_int8 = fmt == LB_FMT_INT8;
  float acc = 0.f;
  for (int kk = lane; kk < k; kk += 32) {
    const int64_t e = int64_t(nn) * k + kk;
    float w;
    if (fmt == LB_FMT_FP16) {
      w = __half2float(reinterpret_cast<const __half *>(codes)[e]);
    } else if (per_row_int8) {
      w = float(int8_t(codes[e])) * __half2float(scales[e / group]);  // exact code * scale (fp32)
    } else {
      const uint32_t b = codes[e >> 1];
      const uint32_t c = (e & 1) ? (b >> 4) : (b & 15u);
      const __half v = fmt == LB_FMT_INT4 ? __int2half_rn(int(c ^ 8u) - 8) : __float2half_rn(c_nf4[c]);
      w = __half2float(__hmul(v, scales[e / group]));
    }
    acc = fmaf(__half2float(x[int64_t(mm) * k + kk]), w, acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    __half yq = __float2half_rn(acc);
    if (bias) yq = __float2half_rn(__half2float(yq) + __half2float(bias[nn]));
    if (z) {
      float d = 0.f;
      for (int r = 0; r < rank; ++r) d = fmaf(__half2float(z[mm * 32 + r]), __half2float(up[int64_t(nn) * rank + r]), d);
      yq = __float2half_rn(__half2float(yq) + __half2float(__float2half_rn(d)));
    }
    y[int64_t(mm) * n + nn] = yq;
  }
}

// generic z projection for any K
__global__ void lowrank_project_generic_kernel(int m, int k, int rank, const __half *__restrict__ x,
                                               const __half *__restrict__ v, __half *__restrict__ z) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  pdl_launch();
  pdl_wait();
  if (warp >= int64_t(m) * 32) return;
  const int mm = int(warp / 32), r = int(warp % 32);
  float acc = 0.f;
  if (r < rank)
    for (int kk = lane; kk < k; kk += 32)
      acc = fmaf(__half2float(x[int64_t(mm) * k + kk]), __half2float(v[int64_t(r) * k + kk]), acc);
  acc = warp_sum(acc);
  if (lane == 0) z[mm * 32 + r] = __float2half_rn(acc);
}

}  // namespace lowbit

namespace lowbit_host {
using namespace lowbit;

int gemv_elems(int fmt) { return fmt == LB_FMT_INT8 ? 16 : (fmt == LB_FMT_FP16 ? 8 : 32); }

bool gemv_supported(int fmt, int group, int m, int n, int k) {
  const int e = gemv_elems(fmt);
  if (m < 1 || m > 4 || n < 1 || k < e || k % e) return false;
  if (fmt != LB_FMT_FP16 && (group % e)) return false;
  return true;
}

static bool exact_dequant() {
  static int v = -1;
  if (v < 0) {
    const char *s = getenv("LOWBIT_GEMV_FACTORED_SCALE");
    v = (s && s[0] == '1') ? 0 : 1;
  }
  return v == 1;
}

static int prefetch_mode() {
  static int v = -1;
  if (v < 0) {
    const char *s = getenv("LOWBIT_GEMV_PREFETCH");
    v = (s && s[0] == '0') ? 0 : 1;
  }
  return v;
}

template <int FMT, int MT>
static cudaError_t launch_gemv_t(const GemvParams &p, int ctas, int threads, size_t smem, cudaStream_t st) {
  cudaError_t e;
  if (exact_dequant() || FMT == LB_FMT_INT8 || FMT == LB_FMT_FP16) {
    auto kern = gemv_kernel<FMT, MT, true>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    return launch_k(kern, dim3(ctas), dim3(threads), smem, st, p);
  }
  auto kern = gemv_kernel<FMT, MT, false>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return launch_k(kern, dim3(ctas), dim3(threads), smem, st, p);
}

template <int FMT>
static cudaError_t launch_gemv_f(const GemvParams &p, int mt, int ctas, int threads, size_t smem, cudaStream_t st) {
  if (mt == 1) return launch_gemv_t<FMT, 1>(p, ctas, threads, smem, st);
  if (mt == 2) return launch_gemv_t<FMT, 2>(p, ctas, threads, smem, st);
  return launch_gemv_t<FMT, 4>(p, ctas, threads, smem, st);
}

cudaError_t launch_lowrank_project(int m, int k, int rank, const uint16_t *x, const uint16_t *v, uint16_t *z,
                                   cudaStream_t st) {
  const bool vec = k % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(v) & 15u) == 0;
  if (vec)
    return launch_k(lowrank_project_kernel, dim3(32, (m + 7) / 8), dim3(256), 0, st, m, k, rank,
                    reinterpret_cast<const __half *>(x), reinterpret_cast<const __half *>(v),
                    reinterpret_cast<__half *>(z));
  const int64_t warps = int64_t(m) * 32;
  return launch_k(lowrank_project_generic_kernel, dim3(unsigned((warps * 32 + 255) / 256)), dim3(256), 0, st, m, k,
                  rank, reinterpret_cast<const __half *>(x), reinterpret_cast<const __half *>(v),
                  reinterpret_cast<__half *>(z));
}

// Choose slices / warps / rows so that the grid covers the SMs with enough 16-byte loads
// in flight and the K slices of a row stay inside one CTA.
cudaError_t launch_gemv(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                        const uint16_t *scales, const uint16_t *z, const uint16_t *up, int rank, const uint16_t *bias,
                        uint16_t *y, cudaStream_t st) {
  GemvParams p = {};
  p.m = m; p.n = n; p.k = k; p.group = fmt == LB_FMT_FP16 ? k : group;
  p.x = reinterpret_cast<const __half *>(x);
  p.codes = codes;
  p.scales = reinterpret_cast<const __half *>(scales);
  p.z = reinterpret_cast<const __half *>(z);
  p.up = reinterpret_cast<const __half *>(up);
  p.rank = rank;
  p.bias = reinterpret_cast<const __half *>(bias);
  p.y = reinterpret_cast<__half *>(y);
  const int e = gemv_elems(fmt);
  const int chunks = k / e;
  p.nslices = (chunks + 31) / 32;
  p.slice_width = (chunks + p.nslices - 1) / p.nslices;
  p.warps_k = p.nslices < kMaxWarps ? p.nslices : kMaxWarps;
  const int mt = m == 1 ? 1 : (m == 2 ? 2 : 4);
  const int unroll = mt == 1 ? 8 : 4;
  p.row_groups = kMaxWarps / p.warps_k;
  // rows per warp: as many as fit while keeping >= ~2 CTAs per SM worth of work
  int rpw = 16;
  while (rpw > unroll && int64_t((n + p.row_groups * rpw - 1) / (p.row_groups * rpw)) < 2 * 148) rpw -= unroll;
  p.rows_per_warp = rpw;
  while (p.row_groups * p.rows_per_warp > kMaxRowsCta) p.row_groups--;
  p.prefetch = prefetch_mode();
  const int rows_cta = p.row_groups * p.rows_per_warp;
  const int ctas = (n + rows_cta - 1) / rows_cta;
  const int threads = 32 * p.warps_k * p.row_groups;
  size_t smem = size_t(kMaxWarps) * kMaxRowsCta * 4 * sizeof(float);
  if (fmt == LB_FMT_NF4) smem += size_t(kLutWords) * 4;
  switch (fmt) {
    case LB_FMT_INT4: return launch_gemv_f<LB_FMT_INT4>(p, mt, ctas, threads, smem, st);
    case LB_FMT_NF4: return launch_gemv_f<LB_FMT_NF4>(p, mt, ctas, threads, smem, st);
    case LB_FMT_INT8: return launch_gemv_f<LB_FMT_INT8>(p, mt, ctas, threads, smem, st);
    default: return launch_gemv_f<LB_FMT_FP16>(p, mt, ctas, threads, smem, st);
  }
}

cudaError_t launch_linear_generic(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                                  const uint16_t *scales, const uint16_t *z, const uint16_t *up, int rank,
                                  const uint16_t *bias, uint16_t *y, cudaStream_t st) {
  const int64_t warps = int64_t(m) * n;
  const int64_t blocks = (warps * 32 + 255) / 256;
  return launch_k(linear_generic_kernel, dim3(unsigned(blocks)), dim3(256), 0, st, fmt, m, n, k,
                  fmt == LB_FMT_FP16 ? k : group, reinterpret_cast<const __half *>(x), codes,
                  reinterpret_cast<const __half *>(scales), reinterpret_cast<const __half *>(z),
                  reinterpret_cast<const __half *>(up), rank, reinterpret_cast<const __half *>(bias),
                  reinterpret_cast<__half *>(y));
}

}  // namespace lowbit_host
