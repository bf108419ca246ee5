// K2: decode dequant-GEMV for M <= 64 with the rank-r correction in the epilogue.
//
// HBM-bound by design.  Each warp streams 16-row weight groups: lane (g, t) = (lane/4,
// lane%4) issues one 128-bit coalesced load of row g and one of row g+8 per 64-byte
// K block (4 lanes cover a row's 64 contiguous bytes), dequantizes its 32 (4-bit),
// 16 (INT8) or 8 (fp16) elements in registers -- INT4 with lop3 + one exact fp16 op
// per pair, NF4 through a per-lane-replicated 256-entry byte->half2 table in shared
// memory (conflict free), INT8 with byte_perm + one exact fp16 subtract -- and
// multiplies them by the group scale exactly as the reference dequantizes
// (rn16(code * scale), torch_npu_lowbit.py:67-75).  The dequantized registers are
// used directly as the A operand of mma.sync m16n8k16 (fp16 x fp16 products,
// fp32 accumulation); x is the B operand, one activation row per column, so every
// M <= 8 costs the same as M = 1 and the dot product costs no FMA-pipe work.
// The K order inside an MMA is a permutation: each lane's x pairs are loaded once per
// K block in the same order the unpack produces the weight pairs, so no weight
// relayout is needed -- the canonical reference bytes are streamed as they are.
// Partial sums are reduced across the CTA's K-split warps in shared memory and, when
// the K range is split across CTAs, through fp32 partials in the caller's workspace:
// the last CTA of a row set (atomic counter, self-resetting) sums them in a fixed
// order, so results are deterministic.  Epilogue (torch_npu_smollm.py:150-164):
// y = half(acc) (per-row INT8 scale first), half(y + bias), half(y + half(z . U[n]^T)).
// For large weights at up to 16 activation rows the rank-32 projection z = half(x . V^T)
// is computed by the same launch (launch_gemv_fused_z): the first CTAs of the grid each
// reduce one K slice of x . V^T into fp32 partials and count their arrival; the CTAs that
// run an epilogue wait (bounded) for all slices and sum them in slice order.  The GEMV
// of a large weight outlasts that chain, so the projection costs no launch of its own.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>

#include "gemv_frag.cuh"

namespace lowbit {

constexpr int kWarps = 8;
constexpr int kMaxRowGroups = 2;          // 16-row groups per warp
constexpr int kLutWords = 256 * 64;       // NF4 table with a 256-byte entry stride
constexpr int kMaxGemvCounters = 4096;    // arrival counters available in the workspace
constexpr int kZArrive = kMaxGemvCounters - 2;   // fused z: slices done, epilogues done
constexpr int kMaxZSlices = 32;

struct GemvParams {
  int m, n, k, group;
  const __half *x;       // [m, k]
  const uint8_t *codes;  // packed rows, canonical reference layout
  const __half *scales;  // [n, k/group] (unused for FP16)
  const __half *z;       // [m, zs] correction projection half(x . V^T), zero past rank, or null
  const __half *up;      // [n, rank]
  int rank;              // <= zs
  int zs;                // z row stride: rank rounded up to a multiple of 32 (<= 128)
  const __half *resid;   // [m, n] added last (half(y + resid)), or null
  const __half *bias;    // [n] or null
  __half *y;             // [m, n]
  int warps_k;           // warps splitting a CTA's K range (1, 2, 4, 8)
  int wk_shift;          // log2(warps_k)
  int rpw;               // 16-row groups per warp (<= kMaxRowGroups)
  int rows_shift;        // log2(rows per CTA) = log2(16 * (8 / warps_k) * rpw)
  int gpr;               // scale groups per row (1 for FP16)
  int kblocks;           // 64-byte K blocks per row
  int kb_per_split;      // K blocks per CTA (gridDim.y splits)
  float *partial;        // [splits, m, n] fp32 when gridDim.y > 1
  int *counters;         // [gridDim.x] arrival counters (zero between calls)
  int prefetch;
  int gshift;            // log2(group / chunk elements) when that is a power of two, else -1
  // fused projection (zv non-null): V [rank, k]; CTAs with blockIdx.x < zx compute K slice
  // blockIdx.y * zx + blockIdx.x of zx * gridDim.y into zpart [slices][m][32] fp32;
  // counters[kZArrive] counts finished slices, counters[kZArrive + 1] finished epilogues
  // (the last resets both); err receives LB_ERR_TIMEOUT if the wait for z gives up
  const __half *zv;
  int zx;
  float *zpart;
  int *err;
  long long wait_cycles;   // bound of the epilogues' wait for the slices (clock cycles)
  int z_extra;             // test hook: arrivals waited for beyond the slices (0 in use)
};

__device__ __forceinline__ int ld_acquire(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One K slice of z^T = V x^T for up to 8 * NCOL activation rows: warp w owns ranks
// 4w .. 4w + 3, lane l the slice's 16-byte chunks l, l + 32, ...; fp16 products are exact
// and summed in fp32 (lane order, then a butterfly), one partial per (row, rank).
template <int NCOL>
__device__ __forceinline__ void gemv_z_slice(const GemvParams &p) {
  constexpr int MR = 8 * NCOL;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int slices = p.zx * gridDim.y, slice = blockIdx.y * p.zx + blockIdx.x;
  const int chunks = p.k / 8;
  const int c0 = int(int64_t(slice) * chunks / slices), c1 = int(int64_t(slice + 1) * chunks / slices);
  float acc[4][MR];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[r][m] = 0.f;
  for (int c = c0 + lane; c < c1; c += 32) {
    uint4 v[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int rr = 4 * warp + r;
      v[r] = rr < p.rank ? *reinterpret_cast<const uint4 *>(p.zv + int64_t(rr) * p.k + 8 * c) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      if (m >= p.m) break;
      const uint4 xv = *reinterpret_cast<const uint4 *>(p.x + int64_t(m) * p.k + 8 * c);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        fma2_f16_f32(acc[r][m], v[r].x, xv.x);
        fma2_f16_f32(acc[r][m], v[r].y, xv.y);
        fma2_f16_f32(acc[r][m], v[r].z, xv.z);
        fma2_f16_f32(acc[r][m], v[r].w, xv.w);
      }
    }
  }
  float *out = p.zpart + int64_t(slice) * p.m * 32;
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    if (m >= p.m) break;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float sum = warp_sum(acc[r][m]);
      if (lane == 0) out[m * 32 + 4 * warp + r] = sum;
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) atomicAdd(p.counters + kZArrive, 1);
}

// NCOL = 8-column groups of activation rows (M <= 8 NCOL).  Up to 16 columns the x pairs
// of a round are loaded up front and each warp may hold two row groups with two
// accumulator chains; from 32 columns on (batched decode) a warp holds one row group and
// its dequantized fragments are reused across the column groups while x is streamed.
// Reduction buffer: [warps_k][rows_cta][LDC] floats, warps_k * rows_cta <= 128 * row groups.
template <int NCOL> constexpr int red_words() { return 128 * (NCOL > 2 ? 1 : kMaxRowGroups) * 8 * NCOL; }

// GS (one activation row, 4-bit formats, group 64 or 128): the codes are decoded without
// their scale, every m16n8k16 tile lies inside one scale group, each group's tiles start a
// fresh fp32 partial (zero accumulator) and the group scale multiplies that partial --
// one FFMA per group and row instead of one fp16 multiply per weight pair.  The products
// code * x are exact in fp32, so the result differs from the reference's
// sum(rn16(code * scale) * x) only by the fp16 rounding of each code * scale.
template <int FMT, int NCOL, int GS = 0>
__global__ void __launch_bounds__(256) gemv_kernel(const GemvParams p) {
  static_assert(GS == 0 || (NCOL == 1 && (FMT == LB_FMT_INT4 || FMT == LB_FMT_NF4) && (GS == 64 || GS == 128)),
                "group-scaled accumulation is for one activation row of 4-bit codes, group 64 or 128");
  constexpr int E = FmtTraits<FMT>::E;
  constexpr int NP = E / 2;          // pairs per lane chunk
  constexpr int TILES = NP / 2;      // m16n8k16 tiles per K block
  constexpr bool kScaled4 = FMT == LB_FMT_INT4 || FMT == LB_FMT_NF4;
  constexpr bool kWide = NCOL > 2;
  constexpr int RG = kWide ? 1 : kMaxRowGroups;   // row groups a warp can hold
  constexpr int CH = kWide ? 1 : 2;               // accumulator chains per (row group, column group)
  constexpr int LDC = 8 * NCOL;                   // reduction row stride (columns)
  extern __shared__ __align__(16) uint32_t smem[];
  float *red = reinterpret_cast<float *>(smem);                        // [warps_k][rows_cta][LDC]
  uint32_t *lut = smem + red_words<NCOL>();
  __shared__ int s_last;

  if constexpr (NCOL <= 2) {
    if (p.zv && int(blockIdx.x) < p.zx) {
      pdl_launch();
      pdl_wait();
      gemv_z_slice<NCOL>(p);
      return;
    }
  }
  const int bx = int(blockIdx.x) - (p.zv ? p.zx : 0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int kw = warp & (p.warps_k - 1), rw = warp >> p.wk_shift;
  const int rows_cta = 1 << p.rows_shift;
  const int row0 = bx * rows_cta;
  const int wrow0 = row0 + 16 * p.rpw * rw;   // this warp's first row
  const int64_t row_bytes = int64_t(p.k) * FmtTraits<FMT>::BITS / 8;
  const int chunks = p.k / E;
  const int kb0 = blockIdx.y * p.kb_per_split;
  const int kb1 = min(p.kblocks, kb0 + p.kb_per_split);

  const int groups_per_row = p.gpr;
  const bool per_row_scale = FMT == LB_FMT_INT8 && p.group == p.k;
  // One round of weight loads: two K blocks x rpw row groups x rows g / g+8, with scales.
  // Per-lane bases of row g (row g+8 and the next row group are fixed offsets from it).
  const uint8_t *code_base = p.codes + int64_t(wrow0 + g) * row_bytes + 16 * t;
  const __half *scale_base = p.scales + int64_t(wrow0 + g) * groups_per_row;
  auto load_round = [&](int kbA, uint4 (&q)[2][RG][2], __half2 (&s2)[2][RG][2]) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int kb = kbA + u * p.warps_k;
      const int chunk = kb * 4 + t;
      const bool kvalid = kb < kb1 && chunk < chunks;
      const int gi = p.gshift >= 0 ? chunk >> p.gshift : (chunk * E) / p.group;
#pragma unroll
      for (int r = 0; r < RG; ++r) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = wrow0 + 16 * r + g + 8 * h;
          const bool ok = r < p.rpw && kvalid && row < p.n;
          if constexpr (GS == 64) {
            // the block's two groups (lanes t = 0, 1 and t = 2, 3) and both their scales
            q[u][r][h] = ok ? ldg_nc_v4(code_base + (16 * r + 8 * h) * row_bytes + int64_t(kb) * 64) : make_uint4(0, 0, 0, 0);
            const uint32_t sv = ok ? *reinterpret_cast<const uint32_t *>(scale_base + (16 * r + 8 * h) * groups_per_row + 2 * kb) : 0u;
            s2[u][r][h] = u32_as_h2(sv);
            continue;
          } else if constexpr (GS == 128) {
            q[u][r][h] = ok ? ldg_nc_v4(code_base + (16 * r + 8 * h) * row_bytes + int64_t(kb) * 64) : make_uint4(0, 0, 0, 0);
            const __half sc = ok ? scale_base[(16 * r + 8 * h) * groups_per_row + kb] : __float2half(0.f);
            s2[u][r][h] = __halves2half2(sc, sc);
            continue;
          }
          q[u][r][h] = ok ? ldg_nc_v4(code_base + (16 * r + 8 * h) * row_bytes + int64_t(kb) * 64) : make_uint4(0, 0, 0, 0);
          if constexpr (FMT != LB_FMT_FP16) {
            const __half sc = (ok && !per_row_scale) ? scale_base[(16 * r + 8 * h) * groups_per_row + gi]
                                                     : __float2half(1.f);
            s2[u][r][h] = __halves2half2(sc, sc);
          } else {
            s2[u][r][h] = __float2half2_rn(1.f);
          }
        }
      }
    }
  };
  // Weights and scales never change while the program runs, so the first round is
  // requested before waiting on the predecessor kernel (bit 1 of p.prefetch).
  const int kb_first = kb0 + kw;
  const bool preloaded = (p.prefetch & 2) && kb_first < kb1;
  uint4 q_first[2][RG][2];
  __half2 s_first[2][RG][2];
  if (preloaded) load_round(kb_first, q_first, s_first);

  pdl_launch();
  if ((p.prefetch & 1) && warp == 0) {
    // the rest of the CTA's weight bytes (K blocks past its first round) start moving
    // into L2 as well; lane r covers rows r, r + 32, ...
    const int rows = min(rows_cta, p.n - row0);
    const int kb_rest = (p.prefetch & 2) ? kb0 + 2 * p.warps_k : kb0;
    const int64_t off = int64_t(kb_rest) * 64;
    const int64_t end = int64_t(kb1) * 64 < row_bytes ? int64_t(kb1) * 64 : row_bytes;
    if (end > off && ((end - off) & 15) == 0)
      for (int r = lane; r < rows; r += 32)
        prefetch_l2_bulk(p.codes + int64_t(row0 + r) * row_bytes + off, uint32_t(end - off));
  }
  if (p.up && (p.z || p.zv) && warp == kWarps - 1 && lane == 0 && blockIdx.y == 0) {
    // the correction factor rows of the CTA's epilogue (U is as constant as the codes):
    // in L2 by the time the main loop ends
    const int rows = min(rows_cta, p.n - row0);   // <= 0 for a CTA past the last row
    if (rows > 0) {
      const __half *u0 = p.up + int64_t(row0) * p.rank;
      const uint32_t bytes = uint32_t(rows) * uint32_t(p.rank) * 2u;
      if ((bytes & 15) == 0 && (reinterpret_cast<uintptr_t>(u0) & 15) == 0) prefetch_l2_bulk(u0, bytes);
    }
  }
  if constexpr (FMT == LB_FMT_NF4) {
    fill_nf4_pair_lut<64>(lut);
    __syncthreads();
  }
  pdl_wait();

  const char *lutb = reinterpret_cast<const char *>(lut);
  const uint32_t lane4 = uint32_t(lane) * 4u;

  // two accumulator chains per (row group, column): consecutive MMA tiles alternate, so
  // each waits on the one two tiles back
  float acc[RG][NCOL][CH][4];
#pragma unroll
  for (int r = 0; r < RG; ++r)
#pragma unroll
    for (int c = 0; c < NCOL; ++c)
#pragma unroll
      for (int h = 0; h < CH; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[r][c][h][i] = 0.f;

  // x pairs of a round, then dequant + MMA of its weights.
  auto compute_round = [&](int kbA, const uint4 (&q)[2][RG][2], const __half2 (&s2)[2][RG][2]) {
    const bool scale = kScaled4 || (FMT == LB_FMT_INT8 && !per_row_scale);
    if constexpr (GS != 0) {
      // One activation row.  B column c holds x only at the K positions of scale group c
      // of the block: group 128 -- lanes g == 0 supply x; group 64 -- lanes (0, t < 2) and
      // (1, t >= 2), the lanes whose 32 elements lie in the block's first / second group.
      // So D column c is group c's partial sum: lanes t == 0 hold columns 0 and 1 of rows
      // g and g + 8, every other column stays zero.
      const bool xlane = GS == 128 ? g == 0 : g == (t >> 1);
      uint32_t xr[2][NP];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int kb = kbA + u * p.warps_k;
        const int chunk = kb * 4 + t;
        load_x_pairs<FMT>(p.x, chunk, kb < kb1 && chunk < chunks && xlane, xr[u]);
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (u == 1 && kbA + p.warps_k >= kb1) break;
#pragma unroll
        for (int r = 0; r < RG; ++r) {
          if (r >= p.rpw) break;
          uint32_t a0[NP], a1[NP];
          unpack_chunk<FMT>(q[u][r][0], s2[u][r][0], false, lutb, lane4, a0);
          unpack_chunk<FMT>(q[u][r][1], s2[u][r][1], false, lutb, lane4, a1);
          float d0[4], d1[4];   // two chains (even / odd tiles), each started from zero
#pragma unroll
          for (int j = 0; j < TILES; j += 2) {
            const uint32_t aa[4] = {a0[2 * j], a1[2 * j], a0[2 * j + 1], a1[2 * j + 1]};
            const uint32_t ab[4] = {a0[2 * j + 2], a1[2 * j + 2], a0[2 * j + 3], a1[2 * j + 3]};
            if (j == 0) {
              mma16816_zero(d0, aa, xr[u][2 * j], xr[u][2 * j + 1]);
              mma16816_zero(d1, ab, xr[u][2 * j + 2], xr[u][2 * j + 3]);
            } else {
              mma16816(d0, aa, xr[u][2 * j], xr[u][2 * j + 1]);
              mma16816(d1, ab, xr[u][2 * j + 2], xr[u][2 * j + 3]);
            }
          }
          const float2 sg = __half22float2(s2[u][r][0]), sg8 = __half22float2(s2[u][r][1]);
          if constexpr (GS == 64) {
            acc[r][0][0][0] = fmaf(d0[1] + d1[1], sg.y, fmaf(d0[0] + d1[0], sg.x, acc[r][0][0][0]));
            acc[r][0][0][2] = fmaf(d0[3] + d1[3], sg8.y, fmaf(d0[2] + d1[2], sg8.x, acc[r][0][0][2]));
          } else {
            acc[r][0][0][0] = fmaf(d0[0] + d1[0], sg.x, acc[r][0][0][0]);
            acc[r][0][0][2] = fmaf(d0[2] + d1[2], sg8.x, acc[r][0][0][2]);
          }
        }
      }
    } else if constexpr (!kWide) {
      uint32_t xr[2][NCOL][NP];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int kb = kbA + u * p.warps_k;
        const int chunk = kb * 4 + t;
        const bool kvalid = kb < kb1 && chunk < chunks;
#pragma unroll
        for (int c = 0; c < NCOL; ++c)
          load_x_pairs<FMT>(p.x + size_t(g + 8 * c) * p.k, chunk, kvalid && g + 8 * c < p.m, xr[u][c]);
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (u == 1 && kbA + p.warps_k >= kb1) break;
#pragma unroll
        for (int r = 0; r < RG; ++r) {
          if (r >= p.rpw) break;
          uint32_t a0[NP], a1[NP];
          unpack_chunk<FMT>(q[u][r][0], s2[u][r][0], scale, lutb, lane4, a0);
          unpack_chunk<FMT>(q[u][r][1], s2[u][r][1], scale, lutb, lane4, a1);
#pragma unroll
          for (int j = 0; j < TILES; ++j) {
            const uint32_t a[4] = {a0[2 * j], a1[2 * j], a0[2 * j + 1], a1[2 * j + 1]};
#pragma unroll
            for (int c = 0; c < NCOL; ++c) mma16816(acc[r][c][j % CH], a, xr[u][c][2 * j], xr[u][c][2 * j + 1]);
          }
        }
      }
    } else {
      // one row group: its dequantized fragments serve every column group in turn
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (u == 1 && kbA + p.warps_k >= kb1) break;
        const int kb = kbA + u * p.warps_k;
        const int chunk = kb * 4 + t;
        const bool kvalid = kb < kb1 && chunk < chunks;
        uint32_t a0[NP], a1[NP];
        unpack_chunk<FMT>(q[u][0][0], s2[u][0][0], scale, lutb, lane4, a0);
        unpack_chunk<FMT>(q[u][0][1], s2[u][0][1], scale, lutb, lane4, a1);
#pragma unroll
        for (int c = 0; c < NCOL; ++c) {
          if (8 * c >= p.m) break;   // column groups past the activation rows
          uint32_t xr[NP];
          load_x_pairs<FMT>(p.x + size_t(g + 8 * c) * p.k, chunk, kvalid && g + 8 * c < p.m, xr);
#pragma unroll
          for (int j = 0; j < TILES; ++j) {
            const uint32_t a[4] = {a0[2 * j], a1[2 * j], a0[2 * j + 1], a1[2 * j + 1]};
            mma16816(acc[0][c][0], a, xr[2 * j], xr[2 * j + 1]);
          }
        }
      }
    }
  };

  // Two K blocks per round: every weight load of the round is in flight before the
  // first dequant, so each warp pays the memory latency once per round.
  if (preloaded) compute_round(kb_first, q_first, s_first);
  for (int kbA = preloaded ? kb_first + 2 * p.warps_k : kb_first; kbA < kb1; kbA += 2 * p.warps_k) {
    uint4 q[2][RG][2];
    __half2 s2[2][RG][2];
    load_round(kbA, q, s2);
    compute_round(kbA, q, s2);
  }

  // C fragment: acc[r][c] = {C[g][2t], C[g][2t+1], C[g+8][2t], C[g+8][2t+1]} with rows =
  // weight rows 16r + {g, g+8}, columns = activation rows 8c + {2t, 2t+1}
#pragma unroll
  for (int r = 0; r < RG; ++r) {
    if (r >= p.rpw) break;
#pragma unroll
    for (int c = 0; c < NCOL; ++c) {
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[i] = acc[r][c][0][i];
#pragma unroll
        for (int h = 1; h < CH; ++h) v[i] += acc[r][c][h][i];
      }
      float *base = red + (kw * rows_cta + 16 * (p.rpw * rw + r)) * LDC + 8 * c + 2 * t;
      base[g * LDC] = v[0];
      base[g * LDC + 1] = v[1];
      base[(g + 8) * LDC] = v[2];
      base[(g + 8) * LDC + 1] = v[3];
    }
  }
  __syncthreads();

  const int splits = gridDim.y;
  const int outs = rows_cta * p.m;
  // sum of the K-split warps' partials of entry (rl, mm), all loads issued first
  auto warp_total = [&](int rl, int mm) {
    float v[kWarps];
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v[w] = w < p.warps_k ? red[(w * rows_cta + rl) * LDC + mm] : 0.f;
    float sum = v[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w)
      if (w < p.warps_k) sum += v[w];
    return sum;
  };
  if (splits > 1) {
    const int64_t mn = int64_t(p.m) * p.n;
    for (int idx = threadIdx.x; idx < outs; idx += blockDim.x) {
      const int mm = idx >> p.rows_shift, rl = idx & (rows_cta - 1), n = row0 + rl;
      if (n >= p.n) continue;
      p.partial[blockIdx.y * mn + int64_t(mm) * p.n + n] = warp_total(rl, mm);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(p.counters + bx, 1) == splits - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int idx = threadIdx.x; idx < outs; idx += blockDim.x) {
      const int mm = idx >> p.rows_shift, rl = idx & (rows_cta - 1), n = row0 + rl;
      if (n >= p.n) continue;
      float v = 0.f;
      for (int sp = 0; sp < splits; ++sp) v += __ldcg(p.partial + sp * mn + int64_t(mm) * p.n + n);
      red[rl * LDC + mm] = v;   // warp-0 slot reused for the total
    }
    if (threadIdx.x == 0) p.counters[bx] = 0;   // ready for the next call
    __syncthreads();
  }

  if (!p.z && !p.zv) {
    // one pass: total (over the K-split warps unless the cross-CTA sum is in slot 0), scale,
    // bias, residual, store
    for (int idx = threadIdx.x; idx < outs; idx += blockDim.x) {
      const int mm = idx >> p.rows_shift, rl = idx & (rows_cta - 1), n = row0 + rl;
      if (n >= p.n) continue;
      float v = splits > 1 ? red[rl * LDC + mm] : warp_total(rl, mm);
      if (per_row_scale) v *= __half2float(p.scales[n]);
      __half yq = __float2half_rn(v);
      if (p.bias) yq = __float2half_rn(__half2float(yq) + __half2float(p.bias[n]));
      if (p.resid) yq = __float2half_rn(__half2float(yq) + __half2float(p.resid[int64_t(mm) * p.n + n]));
      p.y[int64_t(mm) * p.n + n] = yq;
    }
    return;
  }

  // Totals into the warp-0 slot (each thread owns its (row, column) entries).
  if (splits == 1 && p.warps_k > 1) {
    for (int idx = threadIdx.x; idx < outs; idx += blockDim.x) {
      const int mm = idx >> p.rows_shift, rl = idx & (rows_cta - 1);
      red[rl * LDC + mm] = warp_total(rl, mm);   // only this thread reads or writes entry (rl, mm)
    }
    __syncthreads();
  }

  // Correction delta = half(z . U[n]^T) on the tensor cores: per 16-row group, U rows
  // (rank padded to zs with zeros) are the A operand and z (zero beyond the rank) the B
  // operand, zs / 16 m16n8k16 tiles per 8-column group; then
  // y = half(half(half(acc) + bias) + delta) as torch_npu_smollm.py:150-164 stages it, and
  // half(y + residual) when a residual is fused (torch_npu_smollm.py:192).
  const __half *zsrc = p.z;
  int zstride = p.zs;
  if constexpr (NCOL <= 2) {
    __shared__ __align__(16) __half s_z[16 * 32];
    if (p.zv) {
      // wait (bounded) for every K slice of z, then z = half(sum of the slices in order)
      if (threadIdx.x == 0) {
        const int want = p.zx * gridDim.y + p.z_extra;
        if (ld_acquire(p.counters + kZArrive) < want) {
          const long long t0 = clock64();
          while (ld_acquire(p.counters + kZArrive) < want)
            if (clock64() - t0 > p.wait_cycles) { atomicExch(p.err, LB_ERR_TIMEOUT); break; }
        }
      }
      __syncthreads();
      const int slices = p.zx * gridDim.y;
      for (int i = threadIdx.x; i < p.m * 32; i += blockDim.x) {
        float sum = 0.f;
        if ((i & 31) < p.rank)
          for (int sl = 0; sl < slices; ++sl) sum += __ldcg(p.zpart + int64_t(sl) * p.m * 32 + i);
        s_z[i] = __float2half_rn(sum);
      }
      __syncthreads();
      // the last epilogue leaves both counters at zero for the next call
      if (threadIdx.x == 0 && atomicAdd(p.counters + kZArrive + 1, 1) == int(gridDim.x) - p.zx - 1) {
        p.counters[kZArrive] = 0;
        p.counters[kZArrive + 1] = 0;
      }
      zsrc = s_z;
      zstride = 32;
    }
  }
  const int ktiles = zstride / 16;
  // even rank and a 4-byte aligned U: factor pairs are read as one word
  const bool u_pairs = (p.rank & 1) == 0 && (reinterpret_cast<uintptr_t>(p.up) & 3) == 0;
  // one (16-row group, 8-column group) tile per warp at a time: a CTA of 16 rows has 8
  // column groups for its 8 warps at 64 activation rows
  const int ncg = (p.m + 7) >> 3 < NCOL ? (p.m + 7) >> 3 : NCOL;
  for (int job = warp; job < (rows_cta >> 4) * ncg; job += kWarps) {
    const int rg = job / ncg, c = job - rg * ncg;
    const int rl0 = rg * 16;
    {
      const int mz = 8 * c + g;   // activation row of this lane's B column
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      // unrolled to the largest z width (128 columns): every k tile's U and z loads are
      // issued together instead of one L2 round trip per tile
#pragma unroll
      for (int kt = 0; kt < 8; ++kt) {
        if (kt >= ktiles) break;
        uint32_t ua[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = row0 + rl0 + g + 8 * (i & 1);
          const int kk = 16 * kt + 2 * t + 8 * (i >> 1);   // even
          const __half *ur = p.up + int64_t(row) * p.rank;
          if (row >= p.n || kk >= p.rank) {
            ua[i] = 0u;
          } else if (u_pairs) {
            ua[i] = *reinterpret_cast<const uint32_t *>(ur + kk);   // U[row][kk], U[row][kk + 1]
          } else {
            const __half lo = ur[kk], hi = kk + 1 < p.rank ? ur[kk + 1] : __float2half(0.f);
            ua[i] = h2_as_u32(__halves2half2(lo, hi));
          }
        }
        uint32_t b0 = 0, b1 = 0;
        if (mz < p.m) {
          const uint32_t *zr = reinterpret_cast<const uint32_t *>(zsrc + int64_t(mz) * zstride);
          b0 = zr[8 * kt + t];
          b1 = zr[8 * kt + t + 4];
        }
        mma16816(d, ua, b0, b1);
      }
      // the tile's per-row scale, bias and residual are all loaded before its first store
      float rs[4], bi[4], re[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int mm = 8 * c + 2 * t + (i & 1), n = row0 + rl0 + g + 8 * (i >> 1);
        const bool ok = n < p.n && mm < p.m;
        rs[i] = (per_row_scale && ok) ? __half2float(p.scales[n]) : 1.f;
        bi[i] = (p.bias && ok) ? __half2float(p.bias[n]) : 0.f;
        re[i] = (p.resid && ok) ? __half2float(p.resid[int64_t(mm) * p.n + n]) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int rl = rl0 + g + 8 * (i >> 1), mm = 8 * c + 2 * t + (i & 1), n = row0 + rl;
        if (n >= p.n || mm >= p.m) continue;
        float v = red[rl * LDC + mm];
        if (per_row_scale) v *= rs[i];
        __half yq = __float2half_rn(v);
        if (p.bias) yq = __float2half_rn(__half2float(yq) + bi[i]);
        yq = __float2half_rn(__half2float(yq) + __half2float(__float2half_rn(d[i])));
        if (p.resid) yq = __float2half_rn(__half2float(yq) + re[i]);
        red[rl * LDC + mm] = __half2float(yq);   // the slot this lane alone read
      }
    }
  }
  // The finished tile goes out after the loop, in coalesced stores: with no global store
  // inside it, nothing orders the next column group's U / z / residual loads behind the
  // previous one's results (y could alias them as far as the compiler knows), so they
  // overlap (measured on B200, at 64 activation rows storing in the loop serialised one L2
  // round trip per column group and per residual element).
  __syncthreads();
  for (int idx = threadIdx.x; idx < outs; idx += blockDim.x) {
    const int mm = idx >> p.rows_shift, rl = idx & (rows_cta - 1), n = row0 + rl;
    if (n >= p.n) continue;
    p.y[int64_t(mm) * p.n + n] = __float2half_rn(red[rl * LDC + mm]);
  }
}


// z[m, r] = half(sum_k x[m,k] V[r,k]) for r < rank (zero for rank <= r < zs), row stride zs:
// one CTA per (r, m-tile of up to 8 rows); 8 warps split K, 16-byte loads of V and x.
__global__ void __launch_bounds__(256) lowrank_project_kernel(int m, int k, int rank, int zs, const __half *__restrict__ x,
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
    z[int64_t(m0 + threadIdx.x) * zs + r] = __float2half_rn(r < rank ? s : 0.f);
  }
}

// z[m, c] = half(sum_k x[m,k] V[c,k]) for prefill batches (M > 64): one CTA per MT m16 tiles of
// activation rows (two from 4096 rows on: they share every V load, and at that size the grid
// still fills the device); its kZWarps warps split K in 32-element
// chunks and each computes the 32 x 32 tile with mma.sync m16n8k16 -- x rows as the A
// operand, V rows (the correction factor, zero past the rank) as B.  Lane (g, t) loads 16
// contiguous bytes (elements 8t .. 8t+7 of a chunk) of x rows g, g + 8 (+16 for the second
// tile) and of V rows g + 8 nt: the same K permutation for both operands, so one 16-byte
// load feeds two k16 tiles.  The warps' fp32 partials are summed in a fixed order (shared
// memory [warps][16 MT][33], dynamic).  x is read once; V (rank x K) stays in L1/L2.
constexpr int kZWarps = 16;
template <int MT> constexpr int z_smem_bytes() { return kZWarps * 16 * MT * 33 * 4; }
template <int MT>
__global__ void __launch_bounds__(32 * kZWarps) lowrank_project_mma_kernel(int m, int k, int rank, int zs,
                                                                         const __half *__restrict__ x,
                                                                         const __half *__restrict__ v,
                                                                         __half *__restrict__ z) {
  constexpr int kZRows = 16 * MT;
  extern __shared__ float part[];   // [kZWarps][kZRows][33]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int r0 = blockIdx.x * kZRows;
  const int chunks = k / 32;
  const int c0 = warp * chunks / kZWarps, c1 = (warp + 1) * chunks / kZWarps;
  const __half *xr[2 * MT];
  bool rok[2 * MT];
#pragma unroll
  for (int j = 0; j < 2 * MT; ++j) {   // rows g, g + 8 (, g + 16, g + 24)
    const int row = r0 + g + 8 * j;
    rok[j] = row < m;
    xr[j] = x + int64_t(rok[j] ? row : 0) * k + 8 * t;
  }
  const __half *vr[4];
  bool vok[4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int c = nt * 8 + g;
    vok[nt] = c < rank;
    vr[nt] = v + int64_t(vok[nt] ? c : 0) * k + 8 * t;
  }
  pdl_launch();
  pdl_wait();
  float acc[MT][4][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.f;
  const uint4 zero = make_uint4(0, 0, 0, 0);
#pragma unroll 2
  for (int ch = c0; ch < c1; ++ch) {
    const int e = ch * 32;
    uint4 q[2 * MT], qv[4];
#pragma unroll
    for (int j = 0; j < 2 * MT; ++j) q[j] = rok[j] ? *reinterpret_cast<const uint4 *>(xr[j] + e) : zero;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) qv[nt] = vok[nt] ? *reinterpret_cast<const uint4 *>(vr[nt] + e) : zero;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const uint4 qa = q[2 * mt], qb = q[2 * mt + 1];
      const uint32_t a0[4] = {qa.x, qb.x, qa.y, qb.y};   // k positions 2t, 2t+1 | 2t+8, 2t+9 of tile 0
      const uint32_t a1[4] = {qa.z, qb.z, qa.w, qb.w};   // the same positions of tile 1
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        mma16816(acc[mt][nt], a0, qv[nt].x, qv[nt].y);
        mma16816(acc[mt][nt], a1, qv[nt].z, qv[nt].w);
      }
    }
  }
  float *pw = part + warp * kZRows * 33;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      pw[(16 * mt + g) * 33 + nt * 8 + 2 * t] = acc[mt][nt][0];
      pw[(16 * mt + g) * 33 + nt * 8 + 2 * t + 1] = acc[mt][nt][1];
      pw[(16 * mt + g + 8) * 33 + nt * 8 + 2 * t] = acc[mt][nt][2];
      pw[(16 * mt + g + 8) * 33 + nt * 8 + 2 * t + 1] = acc[mt][nt][3];
    }
  __syncthreads();
  for (int i = threadIdx.x; i < kZRows * zs; i += blockDim.x) {
    const int rr = i / zs, c = i % zs;
    if (r0 + rr >= m) continue;
    float sum = 0.f;
    if (c < 32 && c < rank)
      for (int w = 0; w < kZWarps; ++w) sum += part[(w * kZRows + rr) * 33 + c];
    z[int64_t(r0 + rr) * zs + c] = __float2half_rn(sum);
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
__global__ void lowrank_project_generic_kernel(int m, int k, int rank, int zs, const __half *__restrict__ x,
                                               const __half *__restrict__ v, __half *__restrict__ z) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  pdl_launch();
  pdl_wait();
  if (warp >= int64_t(m) * zs) return;
  const int mm = int(warp / zs), r = int(warp % zs);
  float acc = 0.f;
  if (r < rank)
    for (int kk = lane; kk < k; kk += 32)
      acc = fmaf(__half2float(x[int64_t(mm) * k + kk]), __half2float(v[int64_t(r) * k + kk]), acc);
  acc = warp_sum(acc);
  if (lane == 0) z[int64_t(mm) * zs + r] = __float2half_rn(acc);
}

}  // namespace lowbit

namespace lowbit_host {
using namespace lowbit;

int gemv_elems(int fmt) { return fmt == LB_FMT_INT8 ? 16 : (fmt == LB_FMT_FP16 ? 8 : 32); }

// Decode batches up to 64 activation rows: per 16 weight rows the MMA work grows with M,
// but the weights are still read and dequantized once, which the tcgen05 path (one
// 128-row weight tile per CTA regardless of M) cannot match at these sizes.
bool gemv_supported(int fmt, int group, int m, int n, int k) {
  const int e = gemv_elems(fmt);
  if (m < 1 || m > 64 || n < 1 || k < e || k % e) return false;
  if (fmt != LB_FMT_FP16 && fmt != LB_FMT_INT8 && group % e) return false;
  if (fmt == LB_FMT_INT8 && group != k && group % e) return false;
  return true;
}

// bit 0: L2 prefetch of the CTA's weight bytes past its first round, bit 1: first round
// of weight loads into registers, both before waiting on the predecessor
// (LOWBIT_GEMV_PREFETCH, default 3).
int gemv_prefetch_mode() {
  static int v = -1;
  if (v < 0) {
    const char *s = getenv("LOWBIT_GEMV_PREFETCH");
    v = s ? (atoi(s) & 3) : 3;
  }
  return v;
}

struct GemvPlan { int warps_k, rpw, splits, kb_per_split, ctas_x; };

// Work split over 16-row groups x 64-byte K blocks.  A rough time model: resident CTAs
// must keep ~6 MB of 128-bit loads in flight to cover HBM latency, every extra wave and
// every round of loads per warp repeats the latency, and a cross-CTA K split adds a
// reduction pass.  LOWBIT_GEMV_PLAN="warps_k,rpw,splits" overrides the choice (tuning).
static GemvPlan gemv_plan_search(int fmt, int m, int n, int k);

// Plans are pure functions of the problem: cached per (format, M, N, K) unless a plan is
// forced through the environment.
static GemvPlan gemv_plan(int fmt, int m, int n, int k) {
  if (getenv("LOWBIT_GEMV_PLAN")) return gemv_plan_search(fmt, m, n, k);
  static std::mutex mu;
  static std::unordered_map<uint64_t, GemvPlan> cache;
  const uint64_t key = (uint64_t(fmt) << 60) ^ (uint64_t(m) << 48) ^ (uint64_t(uint32_t(n)) << 24) ^ uint64_t(uint32_t(k));
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const GemvPlan pl = gemv_plan_search(fmt, m, n, k);
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() < 65536) cache.emplace(key, pl);
  return pl;
}

static int ilog2(int v) {
  int s = 0;
  while ((1 << s) < v) ++s;
  return s;
}

// Per-launch constants the kernel would otherwise derive with integer divisions.
static void set_shape_fields(GemvParams &p, int fmt, const GemvPlan &pl) {
  p.wk_shift = ilog2(pl.warps_k);
  p.rows_shift = ilog2(16 * (kWarps / pl.warps_k) * pl.rpw);
  p.gpr = fmt == LB_FMT_FP16 ? 1 : p.k / p.group;
}

static GemvPlan gemv_plan_search(int fmt, int m, int n, int k) {
  const int e = gemv_elems(fmt);
  const int kblocks = (k / e + 3) / 4;
  const int groups = (n + 15) / 16;
  if (kblocks < 1 || groups < 1) return {1, 1, 1, 1, 1};
  int fwk = 0, frpw = 0, fsp = 0;
  if (const char *env = getenv("LOWBIT_GEMV_PLAN")) sscanf(env, "%d,%d,%d", &fwk, &frpw, &fsp);
  // fallback (no candidate passed, e.g. a forced plan the shape cannot take): one row group
  // per warp, 8 per CTA, the whole K range per warp
  GemvPlan best = {1, 1, 1, kblocks, (groups + kWarps - 1) / kWarps};
  double best_cost = 1e30;
  for (int wk = 1; wk <= kWarps; wk *= 2) {
    for (int rpw = 1; rpw <= (m > 16 ? 1 : kMaxRowGroups); rpw *= 2) {
      for (int sp = 1; sp <= 16; sp *= 2) {
        if (fwk && (wk != fwk || rpw != frpw || sp != fsp)) continue;
        if (sp > 1 && ((groups + (kWarps / wk) * rpw - 1) / ((kWarps / wk) * rpw)) > kZArrive) continue;
        const int kbs = (kblocks + sp - 1) / sp;
        if (sp > 1 && kbs < wk) break;
        if (wk > 1 && kbs < wk) continue;
        const int wr = kWarps / wk;
        const int ctas = ((groups + wr * rpw - 1) / (wr * rpw)) * ((kblocks + kbs - 1) / kbs);
        const int loads = rpw * ((kbs + wk - 1) / wk);          // 1 KB warp loads per warp
        const int rounds = ((kbs + wk - 1) / wk + 1) / 2;       // two K blocks per round
        // CTAs resident per SM: the 2-column kernel holds more than 128 registers
        const int per_sm = (m > 8 && m <= 16) ? 1 : 2;
        const double resident = ctas < per_sm * 148 ? ctas : per_sm * 148;
        const double fill = resident * kWarps * loads * 1024.0 / 6.0e6;
        const int waves = (ctas + per_sm * 148 - 1) / (per_sm * 148);
        // small problems are latency-bound: below half the in-flight target more CTAs do
        // not shorten a round (fitted to B200 measurements of the candidate plans)
        double cost = waves * (0.6 * rounds + 0.4 + 0.05 * loads) / (fill < 1.0 ? (fill > 0.5 ? fill : 0.5) : 1.0);
        if (sp > 1) cost += 1.5 + (m > 16 ? m / 16.0 : 0.0);   // partial sums grow with M
        if (cost < best_cost) { best_cost = cost; best = {wk, rpw, (kblocks + kbs - 1) / kbs, kbs, (groups + wr * rpw - 1) / (wr * rpw)}; }
      }
    }
  }
  return best;
}

bool gemv1_supported(int fmt, int group, int m, int n, int k, const void *x, const void *codes, const void *scales,
                     const void *up, int rank);
cudaError_t launch_gemv1(int fmt, int group, int n, int k, const uint16_t *x, const uint8_t *codes,
                         const uint16_t *scales, const uint16_t *z, const uint16_t *down, const uint16_t *up, int rank,
                         const uint16_t *bias, uint16_t *y, int *counters, float *zpart, int *err, cudaStream_t st,
                         bool self_z);
size_t gemv1_zpart_bytes();

size_t gemv_workspace_bytes(int fmt, int m, int n, int k) {
  const GemvPlan pl = gemv_plan(fmt, m, n, k);
  if (pl.splits <= 1) return 0;
  return size_t(pl.splits) * m * n * sizeof(float);
}

// CTAs of one kernel that fit on the device at once (cached per kernel and device).
static int resident_ctas(const void *kern, size_t smem) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const uint64_t key = (uint64_t(reinterpret_cast<uintptr_t>(kern)) << 6) ^ uint64_t(dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int per_sm = 0, sms = 0;
  if (ensure_dyn_smem(kern, int(smem)) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 32 * kWarps, smem) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 0;
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = per_sm * sms;
  return per_sm * sms;
}
template <int FMT, int NCOL> static size_t gemv_smem_v() {
  return size_t(red_words<NCOL>()) * sizeof(float) + (FMT == LB_FMT_NF4 ? size_t(kLutWords) * 4 : 0);
}
template <int FMT> static int resident_ctas_f(int ncol, int gs) {
  if constexpr (FMT == LB_FMT_INT4 || FMT == LB_FMT_NF4) {
    if (ncol == 1 && gs == 64)
      return resident_ctas(reinterpret_cast<const void *>(gemv_kernel<FMT, 1, 64>), gemv_smem_v<FMT, 1>());
    if (ncol == 1 && gs == 128)
      return resident_ctas(reinterpret_cast<const void *>(gemv_kernel<FMT, 1, 128>), gemv_smem_v<FMT, 1>());
  }
  return ncol == 1 ? resident_ctas(reinterpret_cast<const void *>(gemv_kernel<FMT, 1>), gemv_smem_v<FMT, 1>())
                   : resident_ctas(reinterpret_cast<const void *>(gemv_kernel<FMT, 2>), gemv_smem_v<FMT, 2>());
}

// Group-scaled accumulation (gemv_kernel's GS) applies to one activation row of INT4 / NF4
// codes with group 64 (K a multiple of 128 and 4-byte aligned scales: two groups' scales
// are read as one word) or 128.  LOWBIT_GEMV_GS=0 turns it off (comparison).
static int gemv_gs(int fmt, int group, int m, int k, const void *scales) {
  static int enabled = -1;
  if (enabled < 0) {
    const char *e = getenv("LOWBIT_GEMV_GS");
    enabled = (e && e[0] == '0') ? 0 : 1;
  }
  if (!enabled || m != 1 || (fmt != LB_FMT_INT4 && fmt != LB_FMT_NF4)) return 0;
  if (group == 64 && k % 128 == 0 && (reinterpret_cast<uintptr_t>(scales) & 3u) == 0) return 64;
  if (group == 128) return 128;
  return 0;
}

// Activation rows and weight bytes from which the projection is fused into the GEMV
// launch (measured on B200: from ~4 MB of codes the GEMV outlasts the slice chain; below
// it the separate projection launch, which overlaps the GEMV's weight preload, is faster).
constexpr int kFuseZMaxRows = 16;
constexpr int64_t kFuseZMinBytes = int64_t(4) << 20;

// Test hook (lb_test_wait_override): the fused projection's wait bound and a number of
// arrivals that no launch makes, so that a test can make the wait run out.
std::atomic<long long> g_wait_cycles{kWaitCycles};
std::atomic<int> g_z_extra{0};

void set_wait_override(long long cycles, int missing) {
  g_wait_cycles.store(cycles > 0 ? cycles : kWaitCycles);
  g_z_extra.store(missing > 0 ? missing : 0);
}

size_t gemv_fused_zpart_bytes(int m) {
  return m <= kFuseZMaxRows ? std::max(size_t(kMaxZSlices) * m * 32 * sizeof(float), gemv1_zpart_bytes()) : 0;
}

template <int FMT, int NCOL, int GS = 0>
static cudaError_t launch_gemv_t(const GemvParams &p, dim3 grid, size_t, cudaStream_t st) {
  auto kern = gemv_kernel<FMT, NCOL, GS>;
  size_t smem = size_t(red_words<NCOL>()) * sizeof(float);
  if (FMT == LB_FMT_NF4) smem += size_t(kLutWords) * 4;
  cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void *>(kern), int(smem));
  if (e != cudaSuccess) return e;
  return launch_k(kern, grid, dim3(32 * kWarps), smem, st, p);
}

template <int FMT>
static cudaError_t launch_gemv_f(const GemvParams &p, int ncol, dim3 grid, size_t smem, cudaStream_t st, int gs = 0) {
  if constexpr (FMT == LB_FMT_INT4 || FMT == LB_FMT_NF4) {
    if (ncol == 1 && gs == 64) return launch_gemv_t<FMT, 1, 64>(p, grid, smem, st);
    if (ncol == 1 && gs == 128) return launch_gemv_t<FMT, 1, 128>(p, grid, smem, st);
  }
  switch (ncol) {
    case 1: return launch_gemv_t<FMT, 1>(p, grid, smem, st);
    case 2: return launch_gemv_t<FMT, 2>(p, grid, smem, st);
    case 4: return launch_gemv_t<FMT, 4>(p, grid, smem, st);
    default: return launch_gemv_t<FMT, 8>(p, grid, smem, st);
  }
}

// zs: z row stride (rank rounded up to 32; the columns past the rank are written as zero).
cudaError_t launch_lowrank_project(int m, int k, int rank, int zs, const uint16_t *x, const uint16_t *v, uint16_t *z,
                                   cudaStream_t st) {
  const bool vec = k % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(v) & 15u) == 0;
  if (vec && m > 64 && zs == 32 && k % 32 == 0) {
    auto go = [&](auto kern, int rows, int smem) -> cudaError_t {
      const cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void *>(kern), smem);
      if (e != cudaSuccess) return e;
      return launch_k(kern, dim3((m + rows - 1) / rows), dim3(32 * kZWarps), size_t(smem), st, m, k, rank, zs,
                      reinterpret_cast<const __half *>(x), reinterpret_cast<const __half *>(v),
                      reinterpret_cast<__half *>(z));
    };
    return m >= 4096 ? go(lowrank_project_mma_kernel<2>, 32, z_smem_bytes<2>())
                     : go(lowrank_project_mma_kernel<1>, 16, z_smem_bytes<1>());
  }
  if (vec)
    return launch_k(lowrank_project_kernel, dim3(zs, (m + 7) / 8), dim3(256), 0, st, m, k, rank, zs,
                    reinterpret_cast<const __half *>(x), reinterpret_cast<const __half *>(v),
                    reinterpret_cast<__half *>(z));
  const int64_t warps = int64_t(m) * zs;
  return launch_k(lowrank_project_generic_kernel, dim3(unsigned((warps * 32 + 255) / 256)), dim3(256), 0, st, m, k,
                  rank, zs, reinterpret_cast<const __half *>(x), reinterpret_cast<const __half *>(v),
                  reinterpret_cast<__half *>(z));
}

// scratch: gemv_workspace_bytes() of caller memory for fp32 partials; counters: an int
// array of kMaxGemvCounters at a fixed place in the workspace, zero before the first call
// and left at zero by every call.
cudaError_t launch_gemv(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                        const uint16_t *scales, const uint16_t *z, int zs, const uint16_t *up, int rank,
                        const uint16_t *bias, const uint16_t *resid, uint16_t *y, void *scratch, int *counters,
                        cudaStream_t st) {
  // one activation row of 4-bit codes: the one-row kernel (csrc/gemv1.cu)
  if (!resid && zs == 32 && rank <= 32 && gemv1_supported(fmt, group, m, n, k, x, codes, scales, z ? up : nullptr, rank))
    return launch_gemv1(fmt, group, n, k, x, codes, scales, z, nullptr, z ? up : nullptr, rank, bias, y, nullptr, nullptr,
                        nullptr, st, false);
  GemvParams p = {};
  p.m = m; p.n = n; p.k = k; p.group = fmt == LB_FMT_FP16 ? k : group;
  p.x = reinterpret_cast<const __half *>(x);
  p.codes = codes;
  p.scales = reinterpret_cast<const __half *>(scales);
  p.z = reinterpret_cast<const __half *>(z);
  p.up = reinterpret_cast<const __half *>(up);
  p.rank = rank;
  p.zs = zs;
  p.bias = reinterpret_cast<const __half *>(bias);
  p.resid = reinterpret_cast<const __half *>(resid);
  p.y = reinterpret_cast<__half *>(y);
  const GemvPlan pl = gemv_plan(fmt, m, n, k);
  p.warps_k = pl.warps_k;
  p.rpw = pl.rpw;
  set_shape_fields(p, fmt, pl);
  p.kblocks = (k / gemv_elems(fmt) + 3) / 4;
  p.kb_per_split = pl.kb_per_split;
  if (pl.splits > 1) {
    p.partial = static_cast<float *>(scratch);
    p.counters = counters;
  }
  p.prefetch = gemv_prefetch_mode();
  p.gshift = -1;
  {
    const int cpg = p.group / gemv_elems(fmt);   // chunks per scale group
    if (fmt != LB_FMT_FP16 && p.group % gemv_elems(fmt) == 0 && cpg > 0 && (cpg & (cpg - 1)) == 0)
      for (p.gshift = 0; (1 << p.gshift) < cpg; ++p.gshift) {}
  }
  const int ncol = m <= 8 ? 1 : (m <= 16 ? 2 : (m <= 32 ? 4 : 8));
  size_t smem = size_t(kWarps) * 64 * 16 * sizeof(float);
  if (fmt == LB_FMT_NF4) smem += size_t(kLutWords) * 4;
  const dim3 grid(pl.ctas_x, pl.splits);
  const int gs = gemv_gs(fmt, p.group, m, k, scales);
  switch (fmt) {
    case LB_FMT_INT4: return launch_gemv_f<LB_FMT_INT4>(p, ncol, grid, smem, st, gs);
    case LB_FMT_NF4: return launch_gemv_f<LB_FMT_NF4>(p, ncol, grid, smem, st, gs);
    case LB_FMT_INT8: return launch_gemv_f<LB_FMT_INT8>(p, ncol, grid, smem, st);
    default: return launch_gemv_f<LB_FMT_FP16>(p, ncol, grid, smem, st);
  }
}

// The decode GEMV with its rank <= 32 correction projection in the same launch, when the
// problem qualifies (<= kFuseZMaxRows rows, >= kFuseZMinBytes of codes, the whole grid
// resident at once so that the epilogues' wait for the slices always ends); *fused says
// whether it launched.  zpart: gemv_fused_zpart_bytes(m) of workspace; counters as for
// launch_gemv (two more at kZArrive); err: the workspace status word.
cudaError_t launch_gemv_fused_z(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                                const uint16_t *scales, const uint16_t *down, const uint16_t *up, int rank,
                                const uint16_t *bias, uint16_t *y, void *scratch, int *counters, float *zpart,
                                int *err, cudaStream_t st, bool *fused) {
  *fused = false;
  if (rank >= 1 && rank <= 32 && gemv1_supported(fmt, group, m, n, k, x, codes, scales, up, rank)) {
    // the one-row kernel (csrc/gemv1.cu): the projection in the same launch from >= 4 MiB of
    // codes (slice CTAs; measured on B200: faster there, while below it the projection's own
    // launch is faster), unless the grid could not be resident at once
    static const int64_t g1_min = [] {   // LOWBIT_G1_FUSE_MIN: the threshold in code bytes (comparison)
      const char *v = getenv("LOWBIT_G1_FUSE_MIN");
      return v ? int64_t(atoll(v)) : kFuseZMinBytes;
    }();
    // LOWBIT_G1_ZSELF=1: below the threshold, every CTA computes z itself from its staged x
    // (redundant V reads from L2, no wait between CTAs; refused for long K or many CTAs)
    static const bool self_z = [] {
      const char *v = getenv("LOWBIT_G1_ZSELF");
      return v && v[0] == '1';
    }();
    const bool big = int64_t(n) * k / 2 >= g1_min;
    if (big ? (!zpart || !err) : !self_z) return cudaSuccess;
    const cudaError_t e = launch_gemv1(fmt, group, n, k, x, codes, scales, nullptr, down, up, rank, bias, y, counters,
                                       zpart, err, st, !big);
    if (e == cudaErrorNotSupported) return cudaSuccess;
    *fused = true;
    return e;
  }
  const int bits = fmt == LB_FMT_INT8 ? 8 : (fmt == LB_FMT_FP16 ? 16 : 4);
  if (m > kFuseZMaxRows || rank < 1 || rank > 32 || !down || !zpart || !err ||
      int64_t(n) * k * bits / 8 < kFuseZMinBytes)
    return cudaSuccess;
  const GemvPlan pl = gemv_plan(fmt, m, n, k);
  const int ncol = m <= 8 ? 1 : 2;
  const int want = std::min(kMaxZSlices, std::max(1, (k / 8 + 31) / 32));
  const int zx = std::max(1, want / pl.splits);
  const int gs = gemv_gs(fmt, fmt == LB_FMT_FP16 ? k : group, m, k, scales);
  int cap = 0;
  switch (fmt) {
    case LB_FMT_INT4: cap = resident_ctas_f<LB_FMT_INT4>(ncol, gs); break;
    case LB_FMT_NF4: cap = resident_ctas_f<LB_FMT_NF4>(ncol, gs); break;
    case LB_FMT_INT8: cap = resident_ctas_f<LB_FMT_INT8>(ncol, gs); break;
    default: cap = resident_ctas_f<LB_FMT_FP16>(ncol, gs); break;
  }
  if (int64_t(zx + pl.ctas_x) * pl.splits > cap) return cudaSuccess;
  GemvParams p = {};
  p.m = m; p.n = n; p.k = k; p.group = fmt == LB_FMT_FP16 ? k : group;
  p.x = reinterpret_cast<const __half *>(x);
  p.codes = codes;
  p.scales = reinterpret_cast<const __half *>(scales);
  p.zv = reinterpret_cast<const __half *>(down);
  p.zx = zx;
  p.zpart = zpart;
  p.err = err;
  p.wait_cycles = g_wait_cycles.load();
  p.z_extra = g_z_extra.load();
  p.up = reinterpret_cast<const __half *>(up);
  p.rank = rank;
  p.zs = 32;
  p.bias = reinterpret_cast<const __half *>(bias);
  p.y = reinterpret_cast<__half *>(y);
  p.warps_k = pl.warps_k;
  p.rpw = pl.rpw;
  set_shape_fields(p, fmt, pl);
  p.kblocks = (k / gemv_elems(fmt) + 3) / 4;
  p.kb_per_split = pl.kb_per_split;
  if (pl.splits > 1) p.partial = static_cast<float *>(scratch);
  p.counters = counters;
  p.prefetch = gemv_prefetch_mode();
  p.gshift = -1;
  {
    const int cpg = p.group / gemv_elems(fmt);
    if (fmt != LB_FMT_FP16 && p.group % gemv_elems(fmt) == 0 && cpg > 0 && (cpg & (cpg - 1)) == 0)
      for (p.gshift = 0; (1 << p.gshift) < cpg; ++p.gshift) {}
  }
  *fused = true;
  const dim3 grid(pl.ctas_x + zx, pl.splits);
  size_t smem = 0;
  switch (fmt) {
    case LB_FMT_INT4: return launch_gemv_f<LB_FMT_INT4>(p, ncol, grid, smem, st, gs);
    case LB_FMT_NF4: return launch_gemv_f<LB_FMT_NF4>(p, ncol, grid, smem, st, gs);
    case LB_FMT_INT8: return launch_gemv_f<LB_FMT_INT8>(p, ncol, grid, smem, st);
    default: return launch_gemv_f<LB_FMT_FP16>(p, ncol, grid, smem, st);
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
