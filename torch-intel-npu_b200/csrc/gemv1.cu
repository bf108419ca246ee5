// K2a: the decode GEMV for ONE activation row of 4-bit codes (INT4 / NF4) at group 64 or
// 128 -- the single-sequence decode projection of torch_npu_smollm.py:150-164 and the
// M = 1 cells of the low-bit sweep.
//
// HBM-bound.  The weight is cut into units of 16 rows x 64 code bytes (one K block of 128
// elements).  Every CTA owns a contiguous run of 16-row groups (whole rows, so a row's sum
// never leaves the CTA) and deals its units out to its warps in equal contiguous ranges;
// one CTA of 16 warps or two of 8 per SM.  A warp keeps a ring of four units of 128-bit
// loads in flight (lane (g, t) loads 16 bytes of rows g and g + 8 at byte 16 t of the
// block); the first ring and an L2 prefetch of the rest of its range are issued before the
// kernel waits on its predecessor (weights never change while a program runs).  The
// activation row is staged once per CTA in shared memory after the wait.
//
// Per unit each lane decodes its 2 x 32 codes into fp16 pairs -- NF4 through a
// per-lane-replicated byte -> half2 table (one byte_perm + one conflict-free shared load
// per code byte), INT4 with one lop3 per pair and no subtraction: a pair holds 1024 + u
// (low nibble) or 1024 + 16 u (high nibble) for u = code ^ 8, and the offset is removed
// per scale group from the activation sums (sum_lo x * 1032 + sum_hi x * 72, computed when
// x is staged).  The pairs are the A operand of mma.sync m16n8k16 (fp16 products exact,
// fp32 accumulation); B column c carries x only at the K positions of scale group c of the
// block, so D column c is that group's partial sum, which the group scale multiplies in
// fp32 (one FFMA per group and row).  The result differs from the reference's
// sum(rn16(code * scale) * x) only by the fp16 rounding of each code * scale.
//
// A warp's sums of each row group it touched go to shared memory; after one CTA barrier the
// pieces of a row group are added in warp order (deterministic) and a warp runs its
// epilogue: y = half(acc), half(y + bias), half(y + half(z . U[n]^T)).  The rank <= 32
// projection z = half(x . V^T) comes from the launch before (z, lowrank_project_kernel) or,
// for weights of >= 4 MiB (whose main loop outlasts it), from the first CTAs of the same
// launch (zv): each reduces one K slice of x . V^T, fences its partials and counts its
// arrival; the last to arrive publishes z as 32 words in the zeroed counter header.  After
// its main loop a CTA takes those words, or sums the slices itself in slice order once all
// have arrived (the same bits either way); the wait is bounded (LB_ERR_TIMEOUT in the
// status word on expiry).  That launch is used only when the whole grid fits on the device
// at once, so the wait always ends.
#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "gemv_frag.cuh"

namespace lowbit {

constexpr int kG1Ring = 4;                 // units of weight loads in flight per warp
constexpr int kG1Lut = 256 * 64 * 4;       // NF4 byte -> half2 table, 256-byte entry stride (bytes)
constexpr int kG1MaxK = 16384;             // activation row staged in shared memory
constexpr int kG1MaxRowGroups = 1 << 16;   // shared pieces per CTA stay small (<= 16 row groups per slot)
constexpr int kG1Counters = 4096;          // arrival counters in the workspace header
constexpr int kG1Done = kG1Counters - 3;   // in-launch projection: CTAs done with the slices
constexpr int kG1ZArrive = kG1Counters - 2;   //   and slices arrived
constexpr int kG1ZWords = kG1Done - 32;       //   and the projection's 32 words (0 = not written)
constexpr int kG1MaxSlices = 32;
constexpr int kG1SelfMaxK = 4096;           // CTA-local projection (zself): longest K
constexpr int64_t kG1SelfMaxBytes = int64_t(8) << 20;   //   and most V bytes read over all CTAs

struct Gemv1Params {
  int n, k;
  int kbs;               // K blocks (128 elements, 64 code bytes) per row
  int rgs;               // 16-row groups (n / 16)
  int rq, rr;            // row groups per main CTA: rq, one more for the first rr CTAs
  int rmax;              // rq + (rr > 0): the shared piece buffer's row groups
  const __half *x;       // [k]
  const uint8_t *codes;  // [n][k / 2], canonical reference bytes
  const __half *scales;  // [n][k / group]
  const __half *bias;    // [n] or null
  __half *y;             // [n]
  const __half *z;       // [>= rank] projection half(x . V^T) from the caller, or null
  const __half *zv;      // V [rank][k] for the in-launch projection, or null
  const __half *up;      // U [n][rank], or null
  int rank;
  int zx;                // CTAs computing z slices (first in the grid; 0 without zv)
  float *zpart;          // [zx][32] slice partials (fp32)
  int *counters;         // the workspace counters: kG1ZWords.., kG1Done, kG1ZArrive (zero between calls)
  int *err;              // status word (LB_ERR_TIMEOUT)
  long long wait_cycles;
  int z_extra;           // test hook: slice arrivals waited for beyond zx (0 in use)
  int zself;             // 1: every main CTA computes z = half(x . V^T) from its staged x (zx = 0)
};

__device__ __forceinline__ int g1_ld_acquire(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t g1_ld_relaxed(const int *p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void g1_st_relaxed(int *p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int g1_atom_add_acq_rel(int *p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ uint32_t g1_ldg_u32(const void *p) {
  uint32_t r;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t g1_ldg_u16(const void *p) {
  unsigned short r;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t g1_lds(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}
template <int OFF>
__device__ __forceinline__ uint32_t g1_lds_imm(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(a), "n"(OFF) : "memory");
  return v;
}

// One K slice of z^T = V x^T (slice blockIdx.x of zx): warp w < 8 owns ranks 4w .. 4w + 3,
// lane l the slice's 16-byte chunks l, l + 32, ...; fp16 products exact, fp32 sums.  Every
// writer fences its partials before the CTA counts the slice arrived.  The slice that
// arrives last sums the partials in slice order (g1_sum_slices), rounds each to half and
// publishes z[r] as the word ~bits(float(z[r])) in counters[kG1ZWords + r]: a word is 0 until
// written (the header is zero between calls) and never 0 once written (0xffffffff is not the
// float of a half).  It then counts itself done with the main CTAs, so the words it stored
// precede the last CTA's reset.
__device__ __forceinline__ uint32_t g1_sum_slices(const Gemv1Params &p, int r) {
  float v[kG1MaxSlices];   // every partial in flight at once (one L2 round trip), then summed in order
#pragma unroll
  for (int sl = 0; sl < kG1MaxSlices; ++sl) v[sl] = sl < p.zx ? __ldcg(p.zpart + sl * 32 + r) : 0.f;
  float s = 0.f;
#pragma unroll
  for (int sl = 0; sl < kG1MaxSlices; ++sl)
    if (sl < p.zx) s += v[sl];
  const float z = r < p.rank ? __half2float(__float2half_rn(s)) : 0.f;
  return ~__float_as_uint(z);
}

__device__ __forceinline__ void g1_release_z(const Gemv1Params &p);

// s_last: one int of the slice CTA's dynamic shared memory (a static __shared__ variable
// would move the dynamic base that the NF4 table's immediate-offset loads rely on).
__device__ void g1_z_slice(const Gemv1Params &p, int *s_last) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int chunks = p.k >> 3;
  const int c0 = int(int64_t(blockIdx.x) * chunks / p.zx), c1 = int(int64_t(blockIdx.x + 1) * chunks / p.zx);
  if (warp < 8) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    // two chunks per lane and step, all their loads issued before the first product (the
    // chunks still reach each sum in the order c, c + 32, c + 64, ...)
    for (int c = c0 + lane; c < c1; c += 64) {
      const bool two = c + 32 < c1;
      const uint4 zero = make_uint4(0, 0, 0, 0);
      const uint4 xa = *reinterpret_cast<const uint4 *>(p.x + 8 * int64_t(c));
      const uint4 xb = two ? *reinterpret_cast<const uint4 *>(p.x + 8 * int64_t(c + 32)) : zero;
      uint4 va[4], vb[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int rr = 4 * warp + r;
        const __half *vr = p.zv + int64_t(rr) * p.k + 8 * int64_t(c);
        va[r] = rr < p.rank ? ldg_nc_v4(vr) : zero;
        vb[r] = rr < p.rank && two ? ldg_nc_v4(vr + 256) : zero;
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        if (4 * warp + r >= p.rank) break;
        fma2_f16_f32(acc[r], va[r].x, xa.x);
        fma2_f16_f32(acc[r], va[r].y, xa.y);
        fma2_f16_f32(acc[r], va[r].z, xa.z);
        fma2_f16_f32(acc[r], va[r].w, xa.w);
        if (two) {
          fma2_f16_f32(acc[r], vb[r].x, xb.x);
          fma2_f16_f32(acc[r], vb[r].y, xb.y);
          fma2_f16_f32(acc[r], vb[r].z, xb.z);
          fma2_f16_f32(acc[r], vb[r].w, xb.w);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float s = warp_sum(acc[r]);
      if (lane == 0) p.zpart[blockIdx.x * 32 + 4 * warp + r] = s;   // zero past the rank
    }
    if (lane == 0) __threadfence();   // this writer's partials reach L2 before the arrival
  }
  __syncthreads();
  if (threadIdx.x == 0) *s_last = g1_atom_add_acq_rel(p.counters + kG1ZArrive, 1) == p.zx + p.z_extra - 1;
  __syncthreads();
  if (*s_last && threadIdx.x < 32) {
    g1_st_relaxed(p.counters + kG1ZWords + threadIdx.x, g1_sum_slices(p, threadIdx.x));
    __threadfence();   // every lane's word before the done count below
    __syncwarp();
    if (threadIdx.x == 0) g1_release_z(p);
  }
}

// The projection, once per main CTA, by warp 0 into zs[32] (fp32 values of the halves):
// the published words when they are all there, else -- once every slice has arrived -- the
// same sums from the partials (same order, so the same bits).  The wait is bounded: on
// timeout the status word says so and the projection counts 0.
__device__ __forceinline__ void g1_collect_z(const Gemv1Params &p, float *zs) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const int want = p.zx + p.z_extra;
    uint32_t w = g1_ld_relaxed(p.counters + kG1ZWords + lane);
    if (!__all_sync(0xffffffffu, w != 0u)) {
      const long long t0 = clock64();
      while (true) {
        // all slices in, as seen by every lane's own acquire (a warp-uniform decision)
        if (__all_sync(0xffffffffu, g1_ld_acquire(p.counters + kG1ZArrive) >= want)) {
          w = g1_sum_slices(p, lane);
          break;
        }
        w = g1_ld_relaxed(p.counters + kG1ZWords + lane);
        if (__all_sync(0xffffffffu, w != 0u)) break;
        if (__any_sync(0xffffffffu, clock64() - t0 > p.wait_cycles)) {
          if (lane == 0) atomicExch(p.err, LB_ERR_TIMEOUT);
          w = 0u;
          break;
        }
      }
    }
    zs[lane] = w != 0u ? __uint_as_float(~w) : 0.f;
  }
  __syncthreads();
}

// One count per main CTA (after its projection was read) and one from the publishing slice
// (after its words were stored; none when the test hook withholds it): the last leaves the
// words and both counters at zero for the next call.
__device__ __forceinline__ void g1_release_z(const Gemv1Params &p) {
  const int total = int(gridDim.x) - p.zx + (p.z_extra == 0 ? 1 : 0);
  if (g1_atom_add_acq_rel(p.counters + kG1Done, 1) == total - 1) {
#pragma unroll 4
    for (int r = 0; r < 32; ++r) p.counters[kG1ZWords + r] = 0;
    p.counters[kG1ZArrive] = 0;
    p.counters[kG1Done] = 0;
  }
}

// Epilogue of row group rg: lane l holds the fp32 total of row 16 rg + (l >> 1) (both lanes
// of a pair; the pair splits the rank).  zs: the projection (fp32 values of the halves) or
// null; u: this lane's U[n][16 hl .. 16 hl + 15] when the rank is 32 (loaded earlier).
__device__ __forceinline__ void g1_epilogue(const Gemv1Params &p, int rg, float v, const float *zs, const uint4 (&u)[2]) {
  const int lane = threadIdx.x & 31;
  const int rho = lane >> 1, hl = lane & 1;
  const int n = rg * 16 + rho;
  const bool corr = zs != nullptr;
  float d = 0.f;
  if (corr) {
    if (p.rank == 32) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint32_t w4[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 u2 = __half22float2(u32_as_h2(w4[j]));
          d = fmaf(zs[16 * hl + 8 * i + 2 * j], u2.x, d);
          d = fmaf(zs[16 * hl + 8 * i + 2 * j + 1], u2.y, d);
        }
      }
    } else {
      const __half *ur = p.up + int64_t(n) * p.rank;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (16 * hl + i < p.rank) d = fmaf(zs[16 * hl + i], __half2float(ur[16 * hl + i]), d);
    }
    d += __shfl_xor_sync(0xffffffffu, d, 1);
  }
  if (hl == 0) {
    __half yq = __float2half_rn(v);
    if (p.bias) yq = __float2half_rn(__half2float(yq) + __half2float(p.bias[n]));
    if (corr) yq = __float2half_rn(__half2float(yq) + __half2float(__float2half_rn(d)));
    p.y[n] = yq;
  }
}

__device__ __forceinline__ void g1_load_u(const Gemv1Params &p, int rg, uint4 (&u)[2]) {
  const int lane = threadIdx.x & 31;
  const uint4 *u4 = reinterpret_cast<const uint4 *>(p.up + int64_t(rg * 16 + (lane >> 1)) * 32 + 16 * (lane & 1));
  u[0] = ldg_nc_v4(u4);
  u[1] = ldg_nc_v4(u4 + 1);
}

// Weight-load cursor of a warp: lane base of row g of the current unit (row g + 8 is 8 rows
// on), its scale base, and the unit's K block.
struct G1Cursor {
  const uint8_t *pl;
  const __half *sl;
  int kb;
};

template <int GS>
__device__ __forceinline__ void g1_load(const Gemv1Params &p, G1Cursor &c, uint4 (&q)[2], uint32_t (&sc)[2],
                                        int64_t rb, int64_t row8, int64_t srow8, int64_t gpr) {
  q[0] = ldg_nc_v4(c.pl);
  q[1] = ldg_nc_v4(c.pl + row8);
  if constexpr (GS == 64) {
    sc[0] = g1_ldg_u32(c.sl);
    sc[1] = g1_ldg_u32(c.sl + srow8);
  } else {
    sc[0] = g1_ldg_u16(c.sl);
    sc[1] = g1_ldg_u16(c.sl + srow8);
  }
  c.pl += 64;
  c.sl += 128 / GS;
  if (++c.kb == p.kbs) {   // next row group
    c.kb = 0;
    c.pl += 15 * rb;
    c.sl += 15 * gpr;
  }
}

// The unit loop of warp j: units [u0, u0 + cnt) of its CTA, local row group rg_first on.
// Each row group's 16 sums go to part[(rg * W + j) * 16 ...].  kLutImm >= 0: the NF4 table
// starts at that shared address (the dynamic shared window's base, the same for every
// launch on a device), so a lookup is one byte_perm (code byte * 256 + 4 lane) and one
// load with an immediate offset; -1: the base is added in a register.
template <int FMT, int GS, int W, int kLutImm>
__device__ __forceinline__ void g1_units(const Gemv1Params &p, int u0, int cnt, int rg_first, G1Cursor &cur,
                                         uint4 (&q)[kG1Ring][2], uint32_t (&sc)[kG1Ring][2], uint32_t s_base,
                                         const float *s_c, float *part, int64_t rb, int64_t row8, int64_t srow8,
                                         int64_t gpr) {
  constexpr bool kNF4 = FMT == LB_FMT_NF4;
  constexpr int kLutBytes = kNF4 ? kG1Lut : 0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  // B operand lanes: group 128 -- lanes g == 0 (all of the block); group 64 -- lanes
  // (0, t < 2) and (1, t >= 2), whose 32 elements lie in the block's first / second group
  const bool xlane = GS == 128 ? g == 0 : g == (t >> 1);
  const uint32_t lane4 = uint32_t(lane) * 4u;
  const uint32_t xs0 = s_base + kLutBytes + 64 * t;   // this lane's 32 activations of block 0
  uint32_t xr[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) xr[i] = 0u;

  float acc0 = 0.f, acc1 = 0.f;   // rows g, g + 8 (lanes t == 0 hold the sums)
  int rg = rg_first, kb = u0 - rg_first * p.kbs;
  uint32_t xa = xs0 + 256 * kb;
  for (int base = 0; base < cnt; base += kG1Ring) {
#pragma unroll
    for (int s = 0; s < kG1Ring; ++s) {
      const int i = base + s;
      if (i >= cnt) break;
      if (xlane) {
#pragma unroll
        for (int v = 0; v < 4; ++v)
          asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(xr[4 * v]), "=r"(xr[4 * v + 1]), "=r"(xr[4 * v + 2]), "=r"(xr[4 * v + 3])
                       : "r"(xa + 16 * v)
                       : "memory");
      }
      float d0[4], d1[4];
      const uint32_t w0[4] = {q[s][0].x, q[s][0].y, q[s][0].z, q[s][0].w};
      const uint32_t w1[4] = {q[s][1].x, q[s][1].y, q[s][1].z, q[s][1].w};
#pragma unroll
      for (int wd = 0; wd < 4; ++wd) {
        uint32_t ta[4], tb[4];   // tiles 2 wd and 2 wd + 1
        if constexpr (kNF4) {
          uint32_t v[8];
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            if constexpr (kLutImm >= 0) {
              v[b] = g1_lds_imm<kLutImm>(__byte_perm(w0[wd], lane4, 0x5504 + 0x10 * b));
              v[4 + b] = g1_lds_imm<kLutImm>(__byte_perm(w1[wd], lane4, 0x5504 + 0x10 * b));
            } else {
              v[b] = g1_lds(s_base + __byte_perm(w0[wd], lane4, 0x5504 + 0x10 * b));
              v[4 + b] = g1_lds(s_base + __byte_perm(w1[wd], lane4, 0x5504 + 0x10 * b));
            }
          }
          // pairs (e0 e1) (e2 e3) | (e4 e5) (e6 e7) of rows g and g + 8
          ta[0] = v[0]; ta[1] = v[4]; ta[2] = v[1]; ta[3] = v[5];
          tb[0] = v[2]; tb[1] = v[6]; tb[2] = v[3]; tb[3] = v[7];
        } else {
          const uint32_t lo_mask = 0x000F000Fu, hi_mask = 0x00F000F0u;
          const uint32_t lo_bits = 0x64086408u, hi_bits = 0x64806480u;
          const uint32_t x0 = w0[wd], x0s = w0[wd] >> 8, x1 = w1[wd], x1s = w1[wd] >> 8;
          // low nibbles (e0 e4) (e2 e6): 1024 + u; high nibbles (e1 e5) (e3 e7): 1024 + 16 u
          ta[0] = lop3_sel(x0, lo_mask, lo_bits); ta[1] = lop3_sel(x1, lo_mask, lo_bits);
          ta[2] = lop3_sel(x0s, lo_mask, lo_bits); ta[3] = lop3_sel(x1s, lo_mask, lo_bits);
          tb[0] = lop3_sel(x0, hi_mask, hi_bits); tb[1] = lop3_sel(x1, hi_mask, hi_bits);
          tb[2] = lop3_sel(x0s, hi_mask, hi_bits); tb[3] = lop3_sel(x1s, hi_mask, hi_bits);
        }
        if (wd == 0) {
          mma16816_zero(d0, ta, xr[0], xr[1]);
          mma16816_zero(d1, tb, xr[2], xr[3]);
        } else {
          mma16816(d0, ta, xr[4 * wd], xr[4 * wd + 1]);
          mma16816(d1, tb, xr[4 * wd + 2], xr[4 * wd + 3]);
        }
      }
      // group partials of rows g (d[0], d[1]) and g + 8 (d[2], d[3]); columns 0 / 1 =
      // the block's groups (group 64) or column 0 = the block (group 128)
      float pg[4];
      if constexpr (kNF4) {
#pragma unroll
        for (int e = 0; e < 4; ++e) pg[e] = d0[e] + d1[e];
      } else {
        float cA, cB = 0.f;
        if constexpr (GS == 64) {
          const float2 c2 = *reinterpret_cast<const float2 *>(s_c + 2 * kb);
          cA = c2.x;
          cB = c2.y;
        } else {
          cA = s_c[kb];
        }
        pg[0] = fmaf(d1[0], 0.0625f, d0[0]) - cA;
        pg[1] = fmaf(d1[1], 0.0625f, d0[1]) - cB;
        pg[2] = fmaf(d1[2], 0.0625f, d0[2]) - cA;
        pg[3] = fmaf(d1[3], 0.0625f, d0[3]) - cB;
      }
      if constexpr (GS == 64) {
        const float2 s0 = __half22float2(u32_as_h2(sc[s][0])), s1 = __half22float2(u32_as_h2(sc[s][1]));
        acc0 = fmaf(pg[1], s0.y, fmaf(pg[0], s0.x, acc0));
        acc1 = fmaf(pg[3], s1.y, fmaf(pg[2], s1.x, acc1));
      } else {
        acc0 = fmaf(pg[0], __half2float(__ushort_as_half((unsigned short)sc[s][0])), acc0);
        acc1 = fmaf(pg[2], __half2float(__ushort_as_half((unsigned short)sc[s][1])), acc1);
      }
      if (i + kG1Ring < cnt) g1_load<GS>(p, cur, q[s], sc[s], rb, row8, srow8, gpr);

      // end of a row group or of the range: this warp's piece of the row group
      ++kb;
      xa += 256;
      if (kb == p.kbs || i == cnt - 1) {
        if (t == 0) {
          float *pp = part + (rg * W + warp) * 16;
          pp[g] = acc0;
          pp[g + 8] = acc1;
        }
        acc0 = 0.f;
        acc1 = 0.f;
        if (kb == p.kbs) {
          kb = 0;
          ++rg;
          xa = xs0;
        }
      }
    }
  }
}

// z = half(x . V^T) by one main CTA from the activation row it staged (p.zself): thread t
// owns rank t / W and the x chunks (t % W) + W j, whose products it adds in chunk order
// (V loads issued 8 chunks at a time before the products); the W threads of a rank (lanes of
// one warp) are then summed by shuffles.  INT4 stages x with each 8-chunk permuted
// ([x0 x4 x2 x6 x1 x5 x3 x7]); V's chunk takes the same permutation.  zs[32]: the fp32
// values of the halves (0 past the rank).
template <bool kPermuted, int W>
__device__ __forceinline__ void g1_z_self(const Gemv1Params &p, const uint8_t *xs, float *zs) {
  constexpr int kB = 8;
  const int r = threadIdx.x / W, sub = threadIdx.x % W;
  const int chunks = p.k >> 3;
  float acc = 0.f;
  if (r < p.rank) {
    const __half *vr = p.zv + int64_t(r) * p.k;
    for (int c0 = sub; c0 < chunks; c0 += W * kB) {
      uint4 v[kB];
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        const int ch = c0 + W * b;
        v[b] = ch < chunks ? ldg_nc_v4(vr + 8 * ch) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        const int ch = c0 + W * b;
        if (ch >= chunks) break;
        const uint4 xv = *reinterpret_cast<const uint4 *>(xs + 16 * ch);
        uint4 vv = v[b];
        if constexpr (kPermuted)
          vv = make_uint4(__byte_perm(v[b].x, v[b].z, 0x5410), __byte_perm(v[b].y, v[b].w, 0x5410),
                          __byte_perm(v[b].x, v[b].z, 0x7632), __byte_perm(v[b].y, v[b].w, 0x7632));
        fma2_f16_f32(acc, vv.x, xv.x);
        fma2_f16_f32(acc, vv.y, xv.y);
        fma2_f16_f32(acc, vv.z, xv.z);
        fma2_f16_f32(acc, vv.w, xv.w);
      }
    }
  }
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (sub == 0) zs[r] = r < p.rank ? __half2float(__float2half_rn(acc)) : 0.f;
}

template <int FMT, int GS, int W>
__global__ void __launch_bounds__(32 * W, 16 / W) gemv1_kernel(const Gemv1Params p) {
  static_assert(FMT == LB_FMT_INT4 || FMT == LB_FMT_NF4, "4-bit codes only");
  static_assert(GS == 64 || GS == 128, "group 64 or 128");
  static_assert(W == 8 || W == 16, "8 or 16 warps");
  constexpr bool kNF4 = FMT == LB_FMT_NF4;
  constexpr int kLutBytes = kNF4 ? kG1Lut : 0;
  extern __shared__ __align__(16) uint8_t g1_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // shared layout: [NF4 table] [x staged, k halves] [INT4: per-group offset sums, k / GS
  // floats] [row-group pieces, rmax x W x 16 floats] [the projection, 32 floats]
  float *s_c = reinterpret_cast<float *>(g1_smem + kLutBytes + 2 * p.k);
  float *part = s_c + (kNF4 ? 0 : p.k / GS);

  if (int(blockIdx.x) < p.zx) {
    if (int(threadIdx.x) < p.rank) {   // the slice of V row threadIdx.x (constant) into L2 before the wait
      const int chunks = p.k >> 3;
      const int c0 = int(int64_t(blockIdx.x) * chunks / p.zx), c1 = int(int64_t(blockIdx.x + 1) * chunks / p.zx);
      if (c1 > c0) prefetch_l2_bulk(p.zv + int64_t(threadIdx.x) * p.k + 8 * int64_t(c0), uint32_t(16 * (c1 - c0)));
    }
    pdl_launch();
    pdl_wait();
    g1_z_slice(p, reinterpret_cast<int *>(g1_smem));
    return;
  }

  // this CTA's row groups [rc0, rc0 + nr) and this warp's units of them
  const int c = int(blockIdx.x) - p.zx;
  const int rc0 = c * p.rq + min(c, p.rr);
  const int nr = p.rq + (c < p.rr ? 1 : 0);
  const int units = nr * p.kbs;
  const int uq = units / W, ur = units % W;
  const int u0 = warp * uq + min(warp, ur);
  const int cnt = uq + (warp < ur ? 1 : 0);
  const int rg_first = u0 / p.kbs;           // local row group of the first unit
  const int g = lane >> 2, t = lane & 3;
  const int64_t rb = p.k >> 1;              // code bytes per row
  const int64_t gpr = p.k / GS;             // scale groups per row
  const int64_t row8 = 8 * rb, srow8 = 8 * gpr;
  const int kb0 = u0 - rg_first * p.kbs;
  const int64_t row0 = (int64_t(rc0) + rg_first) * 16 + g;
  G1Cursor cur = {p.codes + row0 * rb + 64 * kb0 + 16 * t, p.scales + row0 * gpr + kb0 * (128 / GS), kb0};
  uint4 q[kG1Ring][2];
  uint32_t sc[kG1Ring][2];
#pragma unroll
  for (int s = 0; s < kG1Ring; ++s)
    if (s < cnt) g1_load<GS>(p, cur, q[s], sc[s], rb, row8, srow8, gpr);
  pdl_launch();
  if (cnt > kG1Ring && lane < 16) {
    // the rest of the warp's range into L2 as well: lane r covers row r of each row group
    int u = u0 + kG1Ring;
    const int u1 = u0 + cnt;
    while (u < u1) {
      const int rg = u / p.kbs, kb = u - rg * p.kbs;
      const int e = min(u1, (rg + 1) * p.kbs);
      prefetch_l2_bulk(p.codes + ((int64_t(rc0) + rg) * 16 + lane) * rb + 64 * kb, uint32_t(64 * (e - u)));
      u = e;
    }
  }
  if (p.zself && threadIdx.x == 32) {
    // this CTA's share of V (constant, like the codes) into L2 before the wait; every CTA reads all of it
    const int64_t total = int64_t(p.rank) * p.k / 8;   // 16-byte chunks
    const int64_t a = total * c / gridDim.x, b = total * (c + 1) / gridDim.x;
    if (b > a) prefetch_l2_bulk(p.zv + 8 * a, uint32_t(16 * (b - a)));
  }
  if (p.up && warp == W - 1 && lane == 0) {
    // the CTA's correction factor rows (as constant as the codes): in L2 for the epilogue
    const uint32_t bytes = uint32_t(nr) * 16u * uint32_t(p.rank) * 2u;
    const __half *u0p = p.up + int64_t(rc0) * 16 * p.rank;
    if ((bytes & 15) == 0 && (reinterpret_cast<uintptr_t>(u0p) & 15) == 0) prefetch_l2_bulk(u0p, bytes);
  }
  if constexpr (kNF4) {
    fill_nf4_pair_lut<64>(reinterpret_cast<uint32_t *>(g1_smem));
  }
  for (int i = threadIdx.x; i < nr * W * 16; i += 32 * W) part[i] = 0.f;
  pdl_wait();

  // stage x: 8-element chunks; INT4 chunks are stored in the order its pairs are decoded
  // ([x0 x4 x2 x6 x1 x5 x3 x7]) with the group's offset sum 1032 * sum(x_even) + 72 * sum(x_odd)
  {
    const int chunks = p.k >> 3;
    for (int c0 = 0; c0 < chunks; c0 += 32 * W) {
      const int ch = c0 + int(threadIdx.x);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (ch < chunks) v = *reinterpret_cast<const uint4 *>(p.x + 8 * int64_t(ch));
      if constexpr (kNF4) {
        if (ch < chunks) *reinterpret_cast<uint4 *>(g1_smem + kLutBytes + 16 * ch) = v;
      } else {
        const uint4 o = make_uint4(__byte_perm(v.x, v.z, 0x5410), __byte_perm(v.y, v.w, 0x5410),
                                   __byte_perm(v.x, v.z, 0x7632), __byte_perm(v.y, v.w, 0x7632));
        if (ch < chunks) *reinterpret_cast<uint4 *>(g1_smem + kLutBytes + 16 * ch) = o;
        const float2 a = __half22float2(u32_as_h2(v.x)), b = __half22float2(u32_as_h2(v.y));
        const float2 cc = __half22float2(u32_as_h2(v.z)), d = __half22float2(u32_as_h2(v.w));
        float se = (a.x + b.x) + (cc.x + d.x), so = (a.y + b.y) + (cc.y + d.y);
#pragma unroll
        for (int o2 = 1; o2 < GS / 8; o2 <<= 1) {
          se += __shfl_xor_sync(0xffffffffu, se, o2);
          so += __shfl_xor_sync(0xffffffffu, so, o2);
        }
        if (ch < chunks && (ch & (GS / 8 - 1)) == 0) s_c[ch / (GS / 8)] = fmaf(1032.f, se, 72.f * so);
      }
    }
  }
  __syncthreads();
  float *zs = part + p.rmax * W * 16;   // [32] the projection
  // the CTA's own projection, while the first weight loads are still in flight
  if (p.zself) g1_z_self<!kNF4, W>(p, g1_smem + kLutBytes, zs);

  if (cnt > 0) {
    const uint32_t s_base = smem_u32(g1_smem);
    if (!kNF4 || s_base != 0x400u)
      g1_units<FMT, GS, W, -1>(p, u0, cnt, rg_first, cur, q, sc, s_base, s_c, part, rb, row8, srow8, gpr);
    else
      g1_units<FMT, GS, W, 0x400>(p, u0, cnt, rg_first, cur, q, sc, s_base, s_c, part, rb, row8, srow8, gpr);
  }
  __syncthreads();
  // the correction: this warp's first U rows in flight while the projection is collected
  const bool corr = p.up && (p.z || p.zv);
  uint4 u[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
  if (corr && p.rank == 32 && warp < nr) g1_load_u(p, rc0 + warp, u);
  if (p.zself) {
    // zs was written before the main loop (the barrier above orders it before the epilogues)
  } else if (p.zv) {
    g1_collect_z(p, zs);
    // the CTA's done count from the last warp, off the path of the epilogues of warps < nr
    if (threadIdx.x == 32 * (W - 1)) g1_release_z(p);
  } else if (corr) {
    if (threadIdx.x < 32) zs[threadIdx.x] = int(threadIdx.x) < p.rank ? __half2float(p.z[threadIdx.x]) : 0.f;
    __syncthreads();
  }
  // each row group's pieces in warp order, then its epilogue
  for (int r = warp; r < nr; r += W) {
    float v = 0.f;
#pragma unroll
    for (int j = 0; j < W; ++j) v += part[(r * W + j) * 16 + (lane >> 1)];
    if (corr && p.rank == 32 && r != warp) g1_load_u(p, rc0 + r, u);
    g1_epilogue(p, rc0 + r, v, corr ? zs : nullptr, u);
  }
}

}  // namespace lowbit

namespace lowbit_host {
using namespace lowbit;

// LOWBIT_GEMV1=0 turns the one-row kernel off (comparison).
static int g1_env(const char *name, int dflt) {
  const char *e = getenv(name);
  return e ? atoi(e) : dflt;
}

static int g1_sms() {
  static int sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!sms[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v < 1) v = 148;
    sms[dev] = v;
  }
  return sms[dev];
}

// One-row 4-bit problems this kernel takes: K a multiple of the 128-element block (and at
// most kG1MaxK), N a multiple of 16, 16-byte aligned rows and
// activations, 4-byte aligned scale pairs at group 64.
bool gemv1_supported(int fmt, int group, int m, int n, int k, const void *x, const void *codes, const void *scales,
                     const void *up, int rank) {
  static const int enabled = g1_env("LOWBIT_GEMV1", 1);
  if (!enabled || m != 1 || (fmt != LB_FMT_INT4 && fmt != LB_FMT_NF4) || (group != 64 && group != 128)) return false;
  if (k % 128 || k > kG1MaxK || n % 16 || n / 16 > kG1MaxRowGroups) return false;
  const uintptr_t a = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(codes);
  if (a & 15u) return false;
  if (group == 64 && (reinterpret_cast<uintptr_t>(scales) & 3u)) return false;
  if (up && rank == 32 && (reinterpret_cast<uintptr_t>(up) & 15u)) return false;
  return true;
}

// Main CTAs and their size (LOWBIT_G1_MODE): "2x8" (default) two CTAs of 8 warps per SM
// when there are at least two row groups per SM slot, else one CTA of 16 warps per SM;
// "1x8" one CTA of 8 warps per SM (the other half of the SM stays free for the next
// launch's CTAs, whose weight loads then overlap this launch); "1x16" one CTA of 16 warps.
struct G1Plan { int w, ctas, rq, rr, rmax; };
static int g1_mode() {
  static const int mode = [] {
    const char *e = getenv("LOWBIT_G1_MODE");
    if (!e) return 0;
    if (e[0] == '1' && e[1] == 'x' && e[2] == '8') return 1;
    if (e[0] == '1' && e[1] == 'x' && e[2] == '1') return 2;
    return 0;
  }();
  return mode;
}
// zx: the projection's slice CTAs, which take SM slots of their own (fewer slices when the
// main CTAs would otherwise have to share row groups).
static G1Plan g1_plan(int rgs, int &zx) {
  const int sms = g1_sms();
  const int mode = g1_mode();
  const bool eight = mode == 1 || (mode == 0 && rgs >= 2 * sms);
  const int cap = (mode == 0 && eight ? 2 : 1) * sms;
  if (zx > 0 && rgs < cap) zx = std::max(1, std::min(zx, cap - rgs));
  const int slots = std::max(1, cap - zx);
  const int ctas = std::max(1, std::min(rgs, slots));
  const int rq = rgs / ctas, rr = rgs % ctas;
  return {eight ? 8 : 16, ctas, rq, rr, rq + (rr ? 1 : 0)};
}

size_t gemv1_zpart_bytes() { return size_t(kG1MaxSlices) * 32 * sizeof(float); }

template <int FMT, int GS, int W>
static size_t g1_smem_bytes(int k, int rmax) {
  return size_t(FMT == LB_FMT_NF4 ? kG1Lut : 0) + 2 * size_t(k) + (FMT == LB_FMT_NF4 ? 0 : size_t(k / GS) * 4) +
         size_t(rmax) * W * 16 * 4 + 32 * 4;
}

template <int FMT, int GS, int W>
static cudaError_t g1_launch(const Gemv1Params &p, int ctas, cudaStream_t st) {
  auto kern = gemv1_kernel<FMT, GS, W>;
  const size_t smem = g1_smem_bytes<FMT, GS, W>(p.k, p.rmax);
  cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void *>(kern), int(smem));
  if (e != cudaSuccess) return e;
  return launch_k(kern, dim3(ctas), dim3(32 * W), smem, st, p);
}

template <int FMT, int GS, int W>
static int g1_resident(int k, int rmax) {
  const void *kern = reinterpret_cast<const void *>(gemv1_kernel<FMT, GS, W>);
  const size_t smem = g1_smem_bytes<FMT, GS, W>(k, rmax);
  if (ensure_dyn_smem(kern, int(smem)) != cudaSuccess) return 0;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 32 * W, smem) != cudaSuccess) return 0;
  return per_sm * g1_sms();
}

// With the in-launch projection every CTA of the grid must be resident at once (checked
// against the occupancy query); otherwise nothing is launched (cudaErrorNotSupported).
template <int FMT, int GS>
static cudaError_t g1_dispatch(const Gemv1Params &p, const G1Plan &pl, cudaStream_t st) {
  const int ctas = pl.ctas + p.zx;
  if (pl.w == 8) {
    if (p.zx && ctas > g1_resident<FMT, GS, 8>(p.k, p.rmax)) return cudaErrorNotSupported;
    return g1_launch<FMT, GS, 8>(p, ctas, st);
  }
  if (p.zx && ctas > g1_resident<FMT, GS, 16>(p.k, p.rmax)) return cudaErrorNotSupported;
  return g1_launch<FMT, GS, 16>(p, ctas, st);
}

extern std::atomic<long long> g_wait_cycles;
extern std::atomic<int> g_z_extra;

// The one-row GEMV.  Correction: z (the caller's projection, [>= rank] halves) and up, or
// down and up with the projection in the same launch (zpart: gemv1_zpart_bytes() of
// workspace, counters: the header's arrival counters, err: its status word).
cudaError_t launch_gemv1(int fmt, int group, int n, int k, const uint16_t *x, const uint8_t *codes,
                         const uint16_t *scales, const uint16_t *z, const uint16_t *down, const uint16_t *up, int rank,
                         const uint16_t *bias, uint16_t *y, int *counters, float *zpart, int *err, cudaStream_t st,
                         bool self_z) {
  Gemv1Params p = {};
  p.n = n; p.k = k;
  p.kbs = k / 128;
  p.rgs = n / 16;
  p.x = reinterpret_cast<const __half *>(x);
  p.codes = codes;
  p.scales = reinterpret_cast<const __half *>(scales);
  p.bias = reinterpret_cast<const __half *>(bias);
  p.y = reinterpret_cast<__half *>(y);
  int zx = 0;
  if (up && down && self_z) {
    p.up = reinterpret_cast<const __half *>(up);
    p.zv = reinterpret_cast<const __half *>(down);
    p.rank = rank;
    p.zself = 1;
  } else if (up && down) {
    p.up = reinterpret_cast<const __half *>(up);
    p.zv = reinterpret_cast<const __half *>(down);
    p.rank = rank;
    p.zpart = zpart;
    p.counters = counters;
    p.err = err;
    p.wait_cycles = g_wait_cycles.load();
    p.z_extra = g_z_extra.load();
    zx = std::min(kG1MaxSlices, std::max(1, k / 256));
  } else if (up && z) {
    p.up = reinterpret_cast<const __half *>(up);
    p.z = reinterpret_cast<const __half *>(z);
    p.rank = rank;
  }
  const G1Plan pl = g1_plan(p.rgs, zx);
  // the CTA-local projection: every CTA reads all of V from L2 and stages it 8 chunks per
  // thread at a time, so it is taken for short K and a bounded total of those reads only
  if (p.zself && (k > kG1SelfMaxK || int64_t(pl.ctas) * rank * k * 2 > kG1SelfMaxBytes)) return cudaErrorNotSupported;
  p.zx = zx;
  p.rq = pl.rq;
  p.rr = pl.rr;
  p.rmax = pl.rmax;
  if (fmt == LB_FMT_NF4)
    return group == 64 ? g1_dispatch<LB_FMT_NF4, 64>(p, pl, st) : g1_dispatch<LB_FMT_NF4, 128>(p, pl, st);
  return group == 64 ? g1_dispatch<LB_FMT_INT4, 64>(p, pl, st) : g1_dispatch<LB_FMT_INT4, 128>(p, pl, st);
}

}  // namespace lowbit_host
