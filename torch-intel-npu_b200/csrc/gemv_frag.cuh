// Fragment-level building blocks shared by the decode GEMV kernels: per-format unpack of
// a lane's 16-byte code chunk into fp16 pairs (the A operand of mma.sync m16n8k16) and
// the matching permuted load of activation pairs (the B operand).
#pragma once
#include "common.cuh"

namespace lowbit {

template <int FMT> struct FmtTraits;
template <> struct FmtTraits<LB_FMT_INT4> { static constexpr int E = 32; static constexpr int BITS = 4; };
template <> struct FmtTraits<LB_FMT_NF4> { static constexpr int E = 32; static constexpr int BITS = 4; };
template <> struct FmtTraits<LB_FMT_INT8> { static constexpr int E = 16; static constexpr int BITS = 8; };
template <> struct FmtTraits<LB_FMT_FP16> { static constexpr int E = 8; static constexpr int BITS = 16; };



__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// d = A . B with a zero accumulator (the C operand is the constant 0): starts a fresh
// partial sum, e.g. one scale group's, without zeroing registers first.
__device__ __forceinline__ void mma16816_zero(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// The lane's 16-byte chunk -> its fp16 pairs, in the format's natural unpack order.
//   INT4: word w -> (e0,e4) (e1,e5) (e2,e6) (e3,e7) of elements 8w..8w+7
//   NF4 : byte b of word w -> (e2b, e2b+1)
//   INT8: word w -> (e0,e2) (e1,e3) of elements 4w..4w+3
//   FP16: natural pairs
// NF4 reads the byte -> half2 table fill_nf4_pair_lut<64> writes (entry e of lane l at
// byte e*256 + 4l): `lut` is the table base and `lane4` = 4 * lane, so one byte_perm
// (code byte into bits 8-15, lane offset into bits 0-7) forms each address and the
// lookup is one conflict-free LDS.
template <int FMT>
__device__ __forceinline__ void unpack_chunk(const uint4 &q, __half2 s2, bool scale, const char *lut, uint32_t lane4,
                                             uint32_t (&p)[FmtTraits<FMT>::E / 2]) {
  const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
  if constexpr (FMT == LB_FMT_INT4 || FMT == LB_FMT_NF4) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      if constexpr (FMT == LB_FMT_INT4) {
        uint32_t o[4];
        int4_word_to_h2(wv[w], o);
#pragma unroll
        for (int j = 0; j < 4; ++j) p[4 * w + j] = o[j];
      } else {
        const uint32_t b = wv[w];
        p[4 * w + 0] = *reinterpret_cast<const uint32_t *>(lut + __byte_perm(b, lane4, 0x5504));
        p[4 * w + 1] = *reinterpret_cast<const uint32_t *>(lut + __byte_perm(b, lane4, 0x5514));
        p[4 * w + 2] = *reinterpret_cast<const uint32_t *>(lut + __byte_perm(b, lane4, 0x5524));
        p[4 * w + 3] = *reinterpret_cast<const uint32_t *>(lut + __byte_perm(b, lane4, 0x5534));
      }
    }
  } else if constexpr (FMT == LB_FMT_INT8) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t o[2];
      int8_word_to_h2(wv[w], o);
      p[2 * w] = o[0];
      p[2 * w + 1] = o[1];
    }
  } else {
#pragma unroll
    for (int w = 0; w < 4; ++w) p[w] = wv[w];
  }
  if (scale) {
#pragma unroll
    for (int i = 0; i < FmtTraits<FMT>::E / 2; ++i) p[i] = h2_as_u32(__hmul2(u32_as_h2(p[i]), s2));  // rn16(code*scale)
  }
}

// x pairs for the lane's chunk, permuted to match unpack_chunk's pair order.
template <int FMT>
__device__ __forceinline__ void load_x_pairs(const __half *xrow, int chunk, bool valid, uint32_t (&xr)[FmtTraits<FMT>::E / 2]) {
  constexpr int E = FmtTraits<FMT>::E;
  uint32_t nat[E / 2];
#pragma unroll
  for (int v = 0; v < E / 8; ++v) {
    const uint4 q = valid ? *reinterpret_cast<const uint4 *>(xrow + size_t(chunk) * E + v * 8) : make_uint4(0, 0, 0, 0);
    nat[v * 4 + 0] = q.x; nat[v * 4 + 1] = q.y; nat[v * 4 + 2] = q.z; nat[v * 4 + 3] = q.w;
  }
  if constexpr (FMT == LB_FMT_INT4) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t A = nat[w * 4 + 0], B = nat[w * 4 + 1], C = nat[w * 4 + 2], D = nat[w * 4 + 3];
      xr[w * 4 + 0] = __byte_perm(A, C, 0x5410);   // (x0, x4)
      xr[w * 4 + 1] = __byte_perm(A, C, 0x7632);   // (x1, x5)
      xr[w * 4 + 2] = __byte_perm(B, D, 0x5410);   // (x2, x6)
      xr[w * 4 + 3] = __byte_perm(B, D, 0x7632);   // (x3, x7)
    }
  } else if constexpr (FMT == LB_FMT_INT8) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t A = nat[w * 2 + 0], B = nat[w * 2 + 1];
      xr[w * 2 + 0] = __byte_perm(A, B, 0x5410);   // (x0, x2)
      xr[w * 2 + 1] = __byte_perm(A, B, 0x7632);   // (x1, x3)
    }
  } else {
#pragma unroll
    for (int i = 0; i < E / 2; ++i) xr[i] = nat[i];
  }
}

}  // namespace lowbit
