// K3: dequant-GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Orientation ("weights as A"): one CTA owns 128 weight rows (the MMA M dimension) and
// BM activation rows (the MMA N dimension, 16..256).  Per 64-wide K stage:
//   * warp 0 (one lane) TMA-loads the packed code tile [128 rows x 32|64 bytes] and the
//     activation tile [BM x 64] fp16 (128-byte swizzle) into one of S stage buffers --
//     fp16 weights are TMA-loaded straight into the stage's A buffer;
//   * warps 2..9 dequantize the codes exactly as the reference does (rn16(code * scale))
//     into one of two K-major 128B-swizzled A buffers (the A ring is decoupled from the
//     TMA ring: an A buffer is busy only from dequant to MMA completion, a TMA stage from
//     the copy's issue on, so two A buffers free the room for a fourth TMA stage);
//   * warp 1 (one lane) issues 4 x tcgen05.mma (M=128, N=BM, K=16, fp16 in, fp32 TMEM
//     accumulate) and commits to the stage's and the A buffer's "empty" barriers.
// The rank-32 correction is a second TMEM accumulator: U tile [128 x 32] and z tile
// [BM x 32] (64-byte swizzle) feed two more MMAs, issued before the main loop (for the
// dequant formats the two tiles are loaded into the last two A buffers, which the dequant
// warps take over once those MMAs complete), so delta = z.U^T lands beside y_q.
// Epilogue (warps 2..5): tcgen05.ld, per-row INT8 scale, y = half(half(acc)+bias),
// y = half(y + half(delta)), stored transposed to y[m, n].
// Split-K (small M): each split writes fp32 partials to the caller's workspace and
// finalize_kernel applies the same epilogue.
// Every TMA load is CTA-local (one CTA's own shared memory).  Every mbarrier wait is bounded: on timeout the
// kernel records LB_ERR_TIMEOUT in the workspace flag, drains and returns.
#include <cuda.h>
#include <cstdlib>

#include "common.cuh"

namespace lowbit {

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *tm, int c0, int c1, uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(mbar)
      : "memory");
}

// UMMA shared-memory descriptor, K-major, swizzled (bits: start>>4 [0,14), LBO>>4 [16,30),
// SBO>>4 [32,46), version 1 at [46,48), layout type at [61,64)).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = uint64_t((saddr & 0x3FFFFu) >> 4);
  d |= uint64_t(1) << 16;
  d |= uint64_t(sbo_bytes >> 4) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(layout) << 61;
  return d;
}
constexpr uint32_t kSwizzle128 = 2, kSwizzle64 = 4;

// instruction descriptor, kind::f16: D f32, A/B f16, both K-major, N>>3 at 17, M>>4 at 24
__host__ __device__ constexpr uint32_t umma_idesc(int m, int n) {
  return (1u << 4) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar) : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int FMT> struct TcFmt;
template <> struct TcFmt<LB_FMT_INT4> { static constexpr int CODE_BYTES = 32; };
template <> struct TcFmt<LB_FMT_NF4> { static constexpr int CODE_BYTES = 32; };
template <> struct TcFmt<LB_FMT_INT8> { static constexpr int CODE_BYTES = 64; };
template <> struct TcFmt<LB_FMT_FP16> { static constexpr int CODE_BYTES = 0; };

template <int BM> struct TcStages { static constexpr int S = BM >= 256 ? 4 : 6; };

template <int FMT, int BM> struct TcLayout {
  static constexpr bool kDeq = FMT != LB_FMT_FP16;
  static constexpr int S = TcStages<BM>::S;          // TMA stages
  static constexpr int SA = kDeq ? (BM >= 256 ? 3 : 2) : S;   // A buffers (fp16 weight tiles ride the TMA stages)
  static constexpr int A_BYTES = 128 * 128;          // 128 rows x 64 fp16
  static constexpr int B_BYTES = BM * 128;           // BM rows x 64 fp16
  static constexpr int C_BYTES = 128 * TcFmt<FMT>::CODE_BYTES;
  static constexpr int A2_BYTES = 128 * 64;          // U tile, 32 fp16 per row
  static constexpr int B2_BYTES = BM * 64;           // z tile
  static constexpr int LUT_BYTES = FMT == LB_FMT_NF4 ? 256 * 32 * 4 : 0;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + SA * A_BYTES;
  // U and z: the last two A buffers for the dequant formats (so that the first stage's
  // dequant need not wait for the correction MMAs), a region of their own for fp16
  static constexpr int ZSLOT = SA - 2;   // first A buffer holding the correction tiles
  static constexpr int OFF_A2 = kDeq ? OFF_A + ZSLOT * A_BYTES : OFF_B + S * B_BYTES;
  static constexpr int OFF_B2 = kDeq ? OFF_A + (ZSLOT + 1) * A_BYTES : OFF_A2 + A2_BYTES;
  static constexpr int OFF_C = (((kDeq ? OFF_B + S * B_BYTES : OFF_B2 + B2_BYTES) + 1023) / 1024) * 1024;
  static constexpr int OFF_LUT = OFF_C + S * C_BYTES;
  static constexpr int OFF_BAR = ((OFF_LUT + LUT_BYTES + 15) / 16) * 16;
  static constexpr int NBARS = 2 * S + 2 * SA + 2;
  static constexpr int BAR_BYTES = NBARS * 8 + 32;
  static constexpr int TOTAL = OFF_BAR + BAR_BYTES + 1024;  // + alignment slack
  static_assert(A2_BYTES <= A_BYTES && B2_BYTES <= A_BYTES, "U and z tiles fit an A buffer");
  static_assert(TOTAL <= 232448, "shared memory per CTA");
};

struct TcParams {
  int m, n, k, group;
  int stages_total;   // k / 64
  int stages_per_split;
  int splits;
  int has_corr;
  int ldy;            // output row stride (elements)
  const __half *scales;
  const __half *bias;
  __half *y;
  float *partial;     // [splits (+1 correction), m, n] fp32 when splits > 1
  int *counters;      // per-output-tile arrival counters (zero between calls)
  int *err;           // workspace error flag
};

__device__ __forceinline__ uint32_t swz128(int row, int chunk) {
  return uint32_t((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

constexpr int kDequantWarps = 16;
constexpr int kStageGroups = kDequantWarps / 8;   // dequant warp groups working on alternate stages
constexpr int kTcThreads = 32 * (2 + kDequantWarps);

template <int FMT, int BM>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_linear_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_z,
                     const TcParams p) {
  using L = TcLayout<FMT, BM>;
  constexpr int S = L::S;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  constexpr int SA = L::SA;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
  // bars: full_tma[S], empty[S] (TMA stages), full_a[SA], empty_a[SA] (A buffers), corr_full, acc_full
  const uint32_t bar_full_tma = smem_u32(bars), bar_empty = smem_u32(bars + S);
  const uint32_t bar_full_a = smem_u32(bars + 2 * S), bar_empty_a = smem_u32(bars + 2 * S + SA);
  const uint32_t bar_corr = smem_u32(bars + 2 * S + 2 * SA), bar_acc = smem_u32(bars + 2 * S + 2 * SA + 1);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + L::NBARS);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * 128, m0 = blockIdx.y * BM;
  const int split = blockIdx.z;
  const int st_begin = split * p.stages_per_split;
  const int st_end = min(p.stages_total, st_begin + p.stages_per_split);
  const int nst = st_end - st_begin;
  // the correction accumulator is computed once per output tile: by split 0
  const bool corr = p.has_corr && split == 0;
  constexpr bool kDequant = FMT != LB_FMT_FP16;
  constexpr uint32_t kCols = BM * 2 <= 32 ? 32 : (BM * 2 <= 64 ? 64 : (BM * 2 <= 128 ? 128 : (BM * 2 <= 256 ? 256 : 512)));

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(bar_full_tma + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int a = 0; a < SA; ++a) {
      mbar_init(bar_full_a + 8 * a, kDequantWarps / kStageGroups);   // one arrive per warp of a group
      mbar_init(bar_empty_a + 8 * a, 1);
    }
    mbar_init(bar_corr, 1);
    mbar_init(bar_acc, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (FMT == LB_FMT_NF4) fill_nf4_pair_lut(reinterpret_cast<uint32_t *>(smem + L::OFF_LUT));
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  pdl_launch();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_acc = tmem, tmem_corr = tmem + BM;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      pdl_wait();
      if (corr) {
        mbar_expect_tx(bar_corr, L::A2_BYTES + L::B2_BYTES);
        tma_load_2d(sbase + L::OFF_A2, &tm_u, 0, n0, bar_corr);
        tma_load_2d(sbase + L::OFF_B2, &tm_z, 0, m0, bar_corr);
      }
      int issued = 0;
      for (int i = 0; i < nst; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait(bar_empty + 8 * s, ph ^ 1, abort_flag)) break;
        const int kst = st_begin + i;
        ++issued;
        mbar_expect_tx(bar_full_tma + 8 * s, (kDequant ? L::C_BYTES : L::A_BYTES) + L::B_BYTES);
        if (kDequant)
          tma_load_2d(sbase + L::OFF_C + s * L::C_BYTES, &tm_w, kst * TcFmt<FMT>::CODE_BYTES, n0, bar_full_tma + 8 * s);
        else
          tma_load_2d(sbase + L::OFF_A + s * L::A_BYTES, &tm_w, kst * 64, n0, bar_full_tma + 8 * s);
        tma_load_2d(sbase + L::OFF_B + s * L::B_BYTES, &tm_x, kst * 64, m0, bar_full_tma + 8 * s);
      }
      if (*abort_flag) {
        // let every copy this thread started land before the CTA can exit
        for (int j = issued > S ? issued - S : 0; j < issued; ++j) mbar_wait_drain(bar_full_tma + 8 * (j % S), (j / S) & 1);
        if (corr) mbar_wait_drain(bar_corr, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(128, BM);
      bool run = true;
      if (corr) {
        run = mbar_wait(bar_corr, 0, abort_flag);
        if (run) {
          tc_fence_after();
          const uint64_t ad = umma_desc(sbase + L::OFF_A2, 512, kSwizzle64);
          const uint64_t bd = umma_desc(sbase + L::OFF_B2, 512, kSwizzle64);
          umma_f16(tmem_corr, ad, bd, idesc, 0u);
          umma_f16(tmem_corr, ad + 2, bd + 2, idesc, 1u);
          if (kDequant) {   // U and z sit in the last two A buffers: hand them to the dequant warps
            umma_commit(bar_empty_a + 8 * L::ZSLOT);
            umma_commit(bar_empty_a + 8 * (L::ZSLOT + 1));
          }
        }
      }
      for (int i = 0; run && i < nst; ++i) {
        const int s = i % S, a = i % SA;
        if (!mbar_wait(bar_full_tma + 8 * s, (i / S) & 1, abort_flag)) break;
        if (kDequant && !mbar_wait(bar_full_a + 8 * a, (i / SA) & 1, abort_flag)) break;
        tc_fence_after();
        const uint64_t ad = umma_desc(sbase + L::OFF_A + a * L::A_BYTES, 1024, kSwizzle128);
        const uint64_t bd = umma_desc(sbase + L::OFF_B + s * L::B_BYTES, 1024, kSwizzle128);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(tmem_acc, ad + 2 * kk, bd + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(bar_empty + 8 * s);
        if (kDequant) umma_commit(bar_empty_a + 8 * a);
      }
      umma_commit(bar_acc);  // fires when every MMA issued above has completed
    }
  } else {
    // --------------------- dequant (mainloop) + epilogue ----------------------
    // kDequantWarps warps in kStageGroups groups of 8: group g dequantizes the stages
    // i = g, g + kStageGroups, ..., so consecutive stages are in flight at once; within a
    // group thread t handles weight row (t % 128) and the ((t / 128) % 2)-th 32-element half
    // of the stage, and every SM sub-partition runs two warps of each group.
    constexpr int kParts = 2, EPP = 64 / kParts;
    const int t = threadIdx.x - 64;
    const int drow = t & 127, part = (t >> 7) & 1, group = t >> 8;
    if (kDequant) {
      const int n = n0 + drow;
      const bool nok = n < p.n;
      const int gpr = p.k / p.group;
      const bool per_row = FMT == LB_FMT_INT8 && p.group == p.k;
      const uint32_t *lut = reinterpret_cast<const uint32_t *>(smem + L::OFF_LUT) + lane;
      // scales for the next kScaleAhead stages are in flight while the current one dequantizes
      constexpr int kScaleAhead = 4;
      __half2 ring[kScaleAhead];
      auto load_scale = [&](int i) -> __half2 {
        if (per_row || !nok || i >= nst) return __float2half2_rn(1.f);
        const __half v = p.scales[int64_t(n) * gpr + ((st_begin + i) * 64 + part * EPP) / p.group];
        return __halves2half2(v, v);
      };
      pdl_wait();
#pragma unroll
      for (int j = 0; j < kScaleAhead; ++j) ring[j] = load_scale(group + kStageGroups * j);
      // uses of A buffer a: the correction tiles (the last two buffers, if any), then the
      // main stages i = a, a + SA, ...
      for (int i = group; i < nst; i += kStageGroups) {
        const int s = i % S, a = i % SA;
        const int first_use = corr && a >= L::ZSLOT ? 1 : 0;
        const __half2 sc = ring[0];
#pragma unroll
        for (int j = 0; j + 1 < kScaleAhead; ++j) ring[j] = ring[j + 1];
        ring[kScaleAhead - 1] = load_scale(i + kStageGroups * kScaleAhead);
        if (!mbar_wait(bar_full_tma + 8 * s, (i / S) & 1, abort_flag)) break;
        const int use = i / SA + first_use;   // the buffer's previous use must have left the tensor cores
        if (use > 0 && !mbar_wait(bar_empty_a + 8 * a, (use - 1) & 1, abort_flag)) break;
        const uint8_t *crow = smem + L::OFF_C + s * L::C_BYTES + drow * TcFmt<FMT>::CODE_BYTES;
        uint8_t *abuf = smem + L::OFF_A + a * L::A_BYTES;
        if constexpr (FMT == LB_FMT_INT4 || FMT == LB_FMT_NF4) {
          constexpr int W = EPP / 8;   // 32-bit code words (8 codes each) of this part
          static_assert(W == 4, "one 16-byte chunk of codes per thread and stage");
          uint32_t wv[W];
          {
            // the code tile arrives 32B-swizzled: chunk c of row r sits at c ^ ((r >> 2) & 1),
            // so the lanes' 16-byte reads (32 consecutive rows) cover all bank groups
            const uint4 c = *reinterpret_cast<const uint4 *>(crow + 16 * (part ^ ((drow >> 2) & 1)));
            wv[0] = c.x; wv[1] = c.y; wv[2] = c.z; wv[3] = c.w;
          }
#pragma unroll
          for (int w = 0; w < W; ++w) {
            uint32_t o[4];
            if constexpr (FMT == LB_FMT_INT4) {
              uint32_t q[4];
              int4_word_to_h2(wv[w], q);   // (e0,e4) (e1,e5) (e2,e6) (e3,e7)
              o[0] = __byte_perm(q[0], q[1], 0x5410);
              o[1] = __byte_perm(q[2], q[3], 0x5410);
              o[2] = __byte_perm(q[0], q[1], 0x7632);
              o[3] = __byte_perm(q[2], q[3], 0x7632);
            } else {
              const uint32_t b = wv[w];
              o[0] = lut[(b << 5) & 0x1FE0u];
              o[1] = lut[(b >> 3) & 0x1FE0u];
              o[2] = lut[(b >> 11) & 0x1FE0u];
              o[3] = lut[(b >> 19) & 0x1FE0u];
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) o[j] = h2_as_u32(__hmul2(u32_as_h2(o[j]), sc));
            *reinterpret_cast<uint4 *>(abuf + swz128(drow, part * W + w)) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        } else {  // INT8: this thread's EPP bytes -> EPP / 8 chunks of 8 halves
          constexpr int V = EPP / 16;
          uint32_t wv[4 * V];
#pragma unroll
          for (int v = 0; v < V; ++v) {
            // 64B-swizzled code tile: chunk c of row r sits at c ^ ((r >> 1) & 3)
            const uint4 c = *reinterpret_cast<const uint4 *>(crow + 16 * ((EPP / 16 * part + v) ^ ((drow >> 1) & 3)));
            wv[4 * v] = c.x; wv[4 * v + 1] = c.y; wv[4 * v + 2] = c.z; wv[4 * v + 3] = c.w;
          }
#pragma unroll
          for (int j = 0; j < 2 * V; ++j) {
            uint32_t a[2], b[2], o[4];
            int8_word_to_h2(wv[2 * j], a);       // (e0,e2) (e1,e3)
            int8_word_to_h2(wv[2 * j + 1], b);   // (e4,e6) (e5,e7)
            o[0] = __byte_perm(a[0], a[1], 0x5410);
            o[1] = __byte_perm(a[0], a[1], 0x7632);
            o[2] = __byte_perm(b[0], b[1], 0x5410);
            o[3] = __byte_perm(b[0], b[1], 0x7632);
            if (!per_row) {
#pragma unroll
              for (int q = 0; q < 4; ++q) o[q] = h2_as_u32(__hmul2(u32_as_h2(o[q]), sc));
            }
            *reinterpret_cast<uint4 *>(abuf + swz128(drow, part * (EPP / 8) + j)) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_full_a + 8 * a);
      }
    } else {
      pdl_wait();
    }

    // ------------------------------- epilogue ---------------------------------
    const bool ok = __all_sync(0xffffffffu, mbar_wait(bar_acc, 0, abort_flag));
    tc_fence_after();
    const int row = 32 * (warp & 3) + lane;          // TMEM lane this warp may access
    // the warps of a TMEM lane quadrant split the BM columns; a 16-column tile stays whole
    constexpr int kQuads = kDequantWarps / 4;   // warps per TMEM lane quadrant
    constexpr int kColGroups = BM / 16 < kQuads ? BM / 16 : (kQuads >= 4 ? 4 : kQuads);   // divides BM / 16
    constexpr int kColsPerWarp = BM / kColGroups;
    const int chalf = (warp - 2) / 4;   // column group (warps past kColGroups idle here)
    const int n = n0 + row;
    float rs = 1.f;
    if (FMT == LB_FMT_INT8 && p.group == p.k && n < p.n) rs = __half2float(p.scales[n]);
    const float bias = (p.bias && n < p.n) ? __half2float(p.bias[n]) : 0.f;
    const int64_t mn = int64_t(p.m) * p.n;
    if (ok) {
      const uint32_t lane_off = uint32_t(32 * (warp & 3)) << 16;
#pragma unroll 1
      for (int c0 = chalf * kColsPerWarp; c0 < (chalf + 1) * kColsPerWarp && c0 < BM; c0 += 16) {
        uint32_t a[16], d[16];
        tmem_ld16(tmem_acc + lane_off + c0, a);
        if (corr) tmem_ld16(tmem_corr + lane_off + c0, d);
        tmem_ld_wait();
        if (n < p.n) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c0 + j;
            if (m >= p.m) break;
            const float v = __uint_as_float(a[j]) * rs;
            if (p.splits > 1) {
              p.partial[split * mn + int64_t(m) * p.n + n] = v;
              if (corr) p.partial[p.splits * mn + int64_t(m) * p.n + n] = __uint_as_float(d[j]);
              continue;
            }
            __half yq = __float2half_rn(v);
            if (p.bias) yq = __float2half_rn(__half2float(yq) + bias);
            if (corr) yq = __float2half_rn(__half2float(yq) + __half2float(__float2half_rn(__uint_as_float(d[j]))));
            p.y[int64_t(m) * p.ldy + n] = yq;
          }
        }
      }
    }
    if (p.splits > 1) {
      // split-K: the last CTA of this output tile to arrive sums the fp32 partials in split
      // order (deterministic) and applies the epilogue; it leaves the counter at zero.
      int *is_last = reinterpret_cast<int *>(const_cast<int *>(abort_flag)) + 1;
      const int tile = blockIdx.y * gridDim.x + blockIdx.x;
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"r"(32 * kDequantWarps));
      if (threadIdx.x == 64) *is_last = atomicAdd(p.counters + tile, 1) == p.splits - 1;
      asm volatile("bar.sync 1, %0;" ::"r"(32 * kDequantWarps));
      if (*is_last) {
        __threadfence();
        // eight output columns at a time: their partial loads are all in flight together
        // (one L2 round trip per eight columns and split instead of one per column), and
        // each column's splits are still summed in split order
        constexpr int kCB = 8;
        const int c_end = min((chalf + 1) * kColsPerWarp, BM);
        for (int cb = chalf * kColsPerWarp; cb < c_end; cb += kCB) {
          float v[kCB], dz[kCB];
#pragma unroll
          for (int j = 0; j < kCB; ++j) v[j] = dz[j] = 0.f;
          const bool any = n < p.n && m0 + cb < p.m;
          if (any) {
            for (int sp = 0; sp < p.splits; ++sp) {
              float part[kCB];
#pragma unroll
              for (int j = 0; j < kCB; ++j) {
                const int m = m0 + cb + j;
                part[j] = (cb + j < c_end && m < p.m) ? __ldcg(p.partial + sp * mn + int64_t(m) * p.n + n) : 0.f;
              }
#pragma unroll
              for (int j = 0; j < kCB; ++j) v[j] += part[j];
            }
            if (p.has_corr) {
#pragma unroll
              for (int j = 0; j < kCB; ++j) {
                const int m = m0 + cb + j;
                dz[j] = (cb + j < c_end && m < p.m) ? __ldcg(p.partial + p.splits * mn + int64_t(m) * p.n + n) : 0.f;
              }
            }
          }
#pragma unroll
          for (int j = 0; j < kCB; ++j) {
            const int m = m0 + cb + j;
            if (!any || cb + j >= c_end || m >= p.m) continue;
            __half yq = __float2half_rn(v[j]);
            if (p.bias) yq = __float2half_rn(__half2float(yq) + bias);
            if (p.has_corr) yq = __float2half_rn(__half2float(yq) + __half2float(__float2half_rn(dz[j])));
            p.y[int64_t(m) * p.ldy + n] = yq;
          }
        }
        if (threadIdx.x == 64) p.counters[tile] = 0;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) atomicExch(p.err, LB_ERR_TIMEOUT);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
  }
}

}  // namespace lowbit

// ------------------------------------ host ------------------------------------------
#include <cudaTypedefs.h>
#include <mutex>

namespace lowbit_host {
using namespace lowbit;

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void *f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// 2-D tensor map: inner extent `inner` elements, `outer` rows, row pitch `pitch` bytes.
static bool make_map(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
                     uint64_t pitch, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tc_supported(int fmt, int group, int m, int n, int k, int rank) {
  if (m < 1 || n < 1 || k < 64 || k % 64) return false;
  if (fmt == LB_FMT_INT4 || fmt == LB_FMT_NF4 || (fmt == LB_FMT_INT8 && group != k))
    if (group % 32) return false;
  if (rank > 0 && (rank > 32 || rank % 8)) return false;
  return true;
}

int tc_block_m(int m) {
  if (const char *env = getenv("LOWBIT_TC_BM")) {   // tuning: force the activation tile width
    const int bm = atoi(env);
    if (bm == 16 || bm == 32 || bm == 64 || bm == 128 || bm == 256) return bm;
  }
  if (m <= 16) return 16;
  if (m <= 32) return 32;
  if (m <= 64) return 64;
  if (m <= 128) return 128;
  return 256;
}

int tc_splits(int m, int n, int k) {
  if (const char *env = getenv("LOWBIT_TC_SPLITS")) {   // tuning: force the K split count
    const int s = atoi(env);
    if (s >= 1 && s <= 16) return s;
  }
  const int bm = tc_block_m(m);
  const int tiles = ((n + 127) / 128) * ((m + bm - 1) / bm);
  const int stages = k / 64;
  int s = 1;
  if (tiles > 4096) return 1;   // the arrival counters live in a fixed 4096-entry region
  // one wave (a CTA per SM) with at least 16 K stages per split: measured on B200 for
  // 8192x2048 / 2048x8192 / 1536x576 at M = 16..128, a second wave or shorter splits cost
  // more in partial sums than they gain
  while (tiles * s * 2 <= 148 && stages / (s * 2) >= 16) s *= 2;
  return s;
}

size_t tc_partial_bytes(int m, int n, int k) {
  const int s = tc_splits(m, n, k);
  return s > 1 ? size_t(s + 1) * m * n * sizeof(float) : 0;  // + one slice for the correction
}
template <int FMT, int BM>
static cudaError_t launch_tc_t(const CUtensorMap &w, const CUtensorMap &x, const CUtensorMap &u, const CUtensorMap &z,
                               const TcParams &p, cudaStream_t st) {
  using L = TcLayout<FMT, BM>;
  auto kern = tc_linear_kernel<FMT, BM>;
  cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void *>(kern), L::TOTAL);
  if (e != cudaSuccess) return e;
  dim3 grid((p.n + 127) / 128, (p.m + BM - 1) / BM, p.splits);
  return launch_k(kern, grid, dim3(kTcThreads), size_t(L::TOTAL), st, w, x, u, z, p);
}

template <int FMT>
static cudaError_t launch_tc_f(int bm, const CUtensorMap &w, const CUtensorMap &x, const CUtensorMap &u,
                               const CUtensorMap &z, const TcParams &p, cudaStream_t st) {
  switch (bm) {
    case 16: return launch_tc_t<FMT, 16>(w, x, u, z, p, st);
    case 32: return launch_tc_t<FMT, 32>(w, x, u, z, p, st);
    case 64: return launch_tc_t<FMT, 64>(w, x, u, z, p, st);
    case 128: return launch_tc_t<FMT, 128>(w, x, u, z, p, st);
    default: return launch_tc_t<FMT, 256>(w, x, u, z, p, st);
  }
}

// y = x . W^T with the reference epilogue.  z (if non-null) is [m, 32] fp16 in device
// memory, up is U [n, rank].  partial: fp32 scratch of tc_partial_bytes(); err: int flag.
cudaError_t launch_tc(int fmt, int group, int m, int n, int k, const uint16_t *x, const uint8_t *codes,
                      const uint16_t *scales, const uint16_t *z, const uint16_t *up, int rank, const uint16_t *bias,
                      uint16_t *y, int ldy, float *partial, int *counters, int *err, cudaStream_t st) {
  const int bm = tc_block_m(m);
  int splits = tc_splits(m, n, k);
  {
    const int per = (k / 64 + splits - 1) / splits;
    splits = (k / 64 + per - 1) / per;
  }
  CUtensorMap tw, tx, tu, tz;
  bool ok;
  if (fmt == LB_FMT_FP16)
    ok = make_map(&tw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, codes, k, n, uint64_t(k) * 2, 64, 128,
                  CU_TENSOR_MAP_SWIZZLE_128B);
  else {
    const uint64_t rb = fmt == LB_FMT_INT8 ? uint64_t(k) : uint64_t(k) / 2;
    ok = make_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, codes, rb, n, rb, fmt == LB_FMT_INT8 ? 64 : 32, 128,
                  fmt == LB_FMT_INT8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
  }
  ok = ok && make_map(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, k, m, uint64_t(k) * 2, 64, bm, CU_TENSOR_MAP_SWIZZLE_128B);
  const bool corr = z != nullptr;
  if (corr) {
    ok = ok && make_map(&tu, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, up, rank, n, uint64_t(rank) * 2, 32, 128,
                        CU_TENSOR_MAP_SWIZZLE_64B);
    ok = ok && make_map(&tz, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, z, 32, m, 64, 32, bm, CU_TENSOR_MAP_SWIZZLE_64B);
  } else {
    tu = tx;
    tz = tx;
  }
  if (!ok) return cudaErrorInvalidValue;
  TcParams p = {};
  p.m = m; p.n = n; p.k = k; p.group = fmt == LB_FMT_FP16 ? k : group;
  p.stages_total = k / 64;
  p.stages_per_split = (p.stages_total + splits - 1) / splits;
  p.splits = (p.stages_total + p.stages_per_split - 1) / p.stages_per_split;  // no empty split
  p.has_corr = corr ? 1 : 0;
  p.ldy = ldy;
  p.scales = reinterpret_cast<const __half *>(scales);
  p.bias = reinterpret_cast<const __half *>(bias);
  p.y = reinterpret_cast<__half *>(y);
  p.partial = partial;
  p.counters = counters;
  p.err = err;
  cudaError_t e;
  switch (fmt) {
    case LB_FMT_INT4: e = launch_tc_f<LB_FMT_INT4>(bm, tw, tx, tu, tz, p, st); break;
    case LB_FMT_NF4: e = launch_tc_f<LB_FMT_NF4>(bm, tw, tx, tu, tz, p, st); break;
    case LB_FMT_INT8: e = launch_tc_f<LB_FMT_INT8>(bm, tw, tx, tu, tz, p, st); break;
    default: e = launch_tc_f<LB_FMT_FP16>(bm, tw, tx, tu, tz, p, st); break;
  }
  return e;
}

}  // namespace lowbit_host
