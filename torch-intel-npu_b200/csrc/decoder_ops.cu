// SmolLM decoder ops around the low-bit projections, following the staged fp16
// rounding of FrozenSmolLayer.reference_cpu (torch_npu_smollm.py:142-193) and
// FrozenSmolIO (torch_npu_smollm_io.py:45-61).  All HBM-bound, one pass each.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"

namespace lowbit {

__device__ __forceinline__ float block_sum(float v, float *sh) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += sh[i];
  return t;
}

__device__ __forceinline__ float block_max(float v, float *sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int i = 0; i < nw; ++i) t = fmaxf(t, sh[i]);
  return t;
}

// RMSNorm (torch_npu_smollm.py:166-168), optionally fused with the residual add that
// precedes it (:184, :192): h = half(x + r) is written back as the new hidden state.
// One CTA per row; the row is kept in registers (dim <= 8 * 8 * blockDim).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __half *__restrict__ x, const __half *__restrict__ res,
                                                      __half *__restrict__ res_out, const __half *__restrict__ gamma,
                                                      __half *__restrict__ out, int dim, float eps) {
  __shared__ float sh[32];
  pdl_launch();
  pdl_wait();
  const int64_t r = blockIdx.x;
  const __half *xr = x + r * dim;
  constexpr int MAXV = 8;  // up to 8 x 8 halves per thread
  float v[MAXV * 8];
  float ss = 0.f;
  const int nvec = dim / 8;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nvec) {
      uint4 a = *reinterpret_cast<const uint4 *>(xr + c * 8);
      const __half *ah = reinterpret_cast<const __half *>(&a);
      if (res) {
        uint4 b = *reinterpret_cast<const uint4 *>(res + r * dim + c * 8);
        const __half *bh = reinterpret_cast<const __half *>(&b);
        uint4 h;
        __half *hh = reinterpret_cast<__half *>(&h);
#pragma unroll
        for (int j = 0; j < 8; ++j) hh[j] = __float2half_rn(__half2float(ah[j]) + __half2float(bh[j]));
        if (res_out) *reinterpret_cast<uint4 *>(res_out + r * dim + c * 8) = h;
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i * 8 + j] = __half2float(hh[j]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i * 8 + j] = __half2float(ah[j]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[i * 8 + j], v[i * 8 + j], ss);
    }
  }
  const float total = block_sum(ss, sh);
  const float inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(total, float(dim)), eps));
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nvec) {
      uint4 g = *reinterpret_cast<const uint4 *>(gamma + c * 8);
      const __half *gh = reinterpret_cast<const __half *>(&g);
      uint4 o;
      __half *oh = reinterpret_cast<__half *>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j) oh[j] = __hmul(__float2half_rn(__fmul_rn(v[i * 8 + j], inv)), gh[j]);
      *reinterpret_cast<uint4 *>(out + r * dim + c * 8) = o;
    }
  }
}

// RoPE in place (torch_npu_smollm.py:174-177): v = half(half(v*cos) + half(rot(v)*sin)),
// rot(v) = cat(-v[hd/2:], v[:hd/2]).  One thread per (token, head, i < hd/2) pair.
__global__ void rope_kernel(__half *__restrict__ q, __half *__restrict__ k, const int32_t *__restrict__ pos,
                            const __half *__restrict__ cos_t, const __half *__restrict__ sin_t, int table_rows,
                            int tokens, int heads, int kv_heads, int hd, int q_stride, int k_stride) {
  pdl_launch();
  pdl_wait();
  const int half_d = hd / 2;
  const int64_t per_tok = int64_t(heads + kv_heads) * half_d;
  const int64_t total = per_tok * tokens;
  for (int64_t id = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; id < total; id += int64_t(gridDim.x) * blockDim.x) {
    const int t = int(id / per_tok);
    const int rem = int(id % per_tok);
    const int h = rem / half_d, i = rem % half_d;
    __half *base = h < heads ? q + int64_t(t) * q_stride + h * hd : k + int64_t(t) * k_stride + (h - heads) * hd;
    const int p = pos[t];
    if (p < 0 || p >= table_rows) continue;
    const __half a = base[i], b = base[i + half_d];
    const __half c0 = cos_t[int64_t(p) * hd + i], s0 = sin_t[int64_t(p) * hd + i];
    const __half c1 = cos_t[int64_t(p) * hd + i + half_d], s1 = sin_t[int64_t(p) * hd + i + half_d];
    base[i] = __hadd(__hmul(a, c0), __hmul(__hneg(b), s0));
    base[i + half_d] = __hadd(__hmul(b, c1), __hmul(a, s1));
  }
}

// KV Select (torch_npu_smollm.py:288-292): cache[b, h, lengths[b], :] = new row.
__global__ void kv_append_kernel(const __half *__restrict__ k, const __half *__restrict__ v, int kv_stride,
                                 __half *__restrict__ kc, __half *__restrict__ vc, const int32_t *__restrict__ lengths,
                                 int batch, int kvh, int hd, int max_pos) {
  pdl_launch();
  pdl_wait();
  const int64_t total = int64_t(batch) * kvh * hd;
  for (int64_t id = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; id < total; id += int64_t(gridDim.x) * blockDim.x) {
    const int b = int(id / (kvh * hd));
    const int rem = int(id % (kvh * hd));
    const int h = rem / hd, i = rem % hd;
    const int p = lengths[b];
    if (p < 0 || p >= max_pos) continue;
    const int64_t dst = ((int64_t(b) * kvh + h) * max_pos + p) * hd + i;
    kc[dst] = k[int64_t(b) * kv_stride + h * hd + i];
    vc[dst] = v[int64_t(b) * kv_stride + h * hd + i];
  }
}

// Optional prologue of the decode attention: RoPE of this step's q and k and the KV append
// (torch_npu_smollm.py:174-177, :288-292) done by the attention CTA that owns the kv head.
struct RopeAppend {
  const __half *k_new, *v_new;   // [B, kv_stride] rows of the new token; null: no prologue
  int kv_stride;
  const __half *cos_t, *sin_t;   // [table_rows, hd]
  int table_rows;
};

// Position splits of one (sequence, kv head): scratch for each split's softmax state.
struct AttnSplit {
  float *part;     // [B * kvh][splits][REP][2 + HD] fp32: running max, sum, unnormalised p.V
  int *counters;   // [B * kvh] arrival counters, zero between calls (the last CTA resets)
};

// (m, l, a) <- the softmax state of two disjoint position sets merged: m the larger max,
// l and a rescaled by exp(m_i - m); an empty set (m = -inf) contributes nothing.
__device__ __forceinline__ float softmax_weight(float mi, float m) { return mi == -INFINITY ? 0.f : expf(mi - m); }

// One-token GQA attention, one pass over the cache (torch_npu_smollm.py:178-182):
// s_j = half(half(q.k_j) * scale) as the reference stages it, then an online softmax --
// each 8-lane group keeps the running max m, sum l = sum_j exp(s_j - m) and
// a = sum_j exp(s_j - m) v_j (fp32) over the rows it reads -- merged across the groups of
// a warp, the warps of the CTA and, when the positions are split across CTAs, the splits
// (the last CTA of a (sequence, kv head) to finish merges them in split order, so the
// result does not depend on timing); out = half(a / l).  The reference rounds
// p_j = exp(s_j - max) / sum to fp16 before p.V; here p stays fp32 (a relative
// difference of at most 2^-11 per term).
// Grid (B * kvh, splits); split s reads positions [s * per, (s + 1) * per), per a
// multiple of 16.  Keys and values are read as 16-byte pieces (8 lanes per 128-byte row,
// 4 rows per warp, 4 rows per lane in flight): a warp step reads the K and V rows of 16
// positions.  The optional prologue (RoPE of q and the new k, KV append) is done by the
// split that owns the appended position -- no other split reads it.
template <int HD, int REP>
// kc / vc are written by the prologue and read back in the same kernel, so they are not
// declared read-only (no non-coherent loads of the appended row).
__global__ void __launch_bounds__(256) attention_decode_kernel(const __half *__restrict__ q, int q_stride,
                                                               __half *kc, __half *vc,
                                                               const int32_t *__restrict__ lengths,
                                                               __half *__restrict__ out, int heads, int kvh,
                                                               int max_pos, float scale, const RopeAppend ra,
                                                               const AttnSplit sp) {
  static_assert(HD == 64, "rows are 8 lanes x 8 halves");
  constexpr int kUnroll = 4;
  constexpr int kWarps = 8;
  constexpr int ST = 2 + HD;   // one softmax state: m, l, a[HD]
  __shared__ float red[kWarps][REP][ST];
  __shared__ int s_last;
  pdl_launch();
  pdl_wait();
  const int bg = blockIdx.x, b = bg / kvh, g = bg % kvh;
  const int split = blockIdx.y, splits = gridDim.y;
  const int pos = lengths[b];
  const int len = min(pos + 1, max_pos);
  const int per = ((len + splits - 1) / splits + 15) & ~15;
  const int j_begin = min(len, split * per), j_end = min(len, j_begin + per);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane >> 3, l8 = lane & 7;
  __half *kbase = kc + (int64_t(b) * kvh + g) * max_pos * HD;
  __half *vbase = vc + (int64_t(b) * kvh + g) * max_pos * HD;
  // RoPE staging v' = half(half(v cos) + half(rot(v) sin)), rot(v) = cat(-v[hd/2:], v[:hd/2]);
  // positions outside the table are left unrotated, as lb_rope does
  const bool rotate = ra.k_new != nullptr && pos >= 0 && pos < ra.table_rows;
  if (ra.k_new != nullptr && pos >= j_begin && pos < j_end) {
    if (threadIdx.x < HD / 2) {
      const int i = threadIdx.x;
      const __half *kn = ra.k_new + int64_t(b) * ra.kv_stride + g * HD;
      const __half *vn = ra.v_new + int64_t(b) * ra.kv_stride + g * HD;
      __half *krow = kbase + int64_t(pos) * HD;
      __half *vrow = vbase + int64_t(pos) * HD;
      __half a = kn[i], c = kn[i + HD / 2];
      if (rotate) {
        const __half *ct = ra.cos_t + int64_t(pos) * HD, *st = ra.sin_t + int64_t(pos) * HD;
        const __half a2 = __hadd(__hmul(a, ct[i]), __hmul(__hneg(c), st[i]));
        c = __hadd(__hmul(c, ct[i + HD / 2]), __hmul(a, st[i + HD / 2]));
        a = a2;
      }
      krow[i] = a;
      krow[i + HD / 2] = c;
      vrow[i] = vn[i];
      vrow[i + HD / 2] = vn[i + HD / 2];
    }
    __syncthreads();   // the appended row is read back below by other threads of this CTA
  }
  float qv[REP][8];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    uint4 qq = *reinterpret_cast<const uint4 *>(q + int64_t(b) * q_stride + (g * REP + r) * HD + l8 * 8);
    if (rotate) {
      // the partner half (element j +- hd/2) lives in lane l8 ^ 4 of the same 8-lane group
      uint4 pp;
      pp.x = __shfl_xor_sync(0xffffffffu, qq.x, 4);
      pp.y = __shfl_xor_sync(0xffffffffu, qq.y, 4);
      pp.z = __shfl_xor_sync(0xffffffffu, qq.z, 4);
      pp.w = __shfl_xor_sync(0xffffffffu, qq.w, 4);
      const __half *qh0 = reinterpret_cast<const __half *>(&qq), *ph = reinterpret_cast<const __half *>(&pp);
      const __half *ct = ra.cos_t + int64_t(pos) * HD + l8 * 8, *st = ra.sin_t + int64_t(pos) * HD + l8 * 8;
      uint4 rq;
      __half *rh = reinterpret_cast<__half *>(&rq);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const __half part = l8 < 4 ? __hneg(ph[e]) : ph[e];
        rh[e] = __hadd(__hmul(qh0[e], ct[e]), __hmul(part, st[e]));
      }
      qq = rq;
    }
    const __half *qh = reinterpret_cast<const __half *>(&qq);
#pragma unroll
    for (int e = 0; e < 8; ++e) qv[r][e] = __half2float(qh[e]);
  }
  // ---- one pass: scores, running max / sum, p.V ------------------------------------
  float m[REP], l[REP], a[REP][8];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) a[r][e] = 0.f;
  }
  for (int j0 = j_begin + warp * 4 * kUnroll; j0 < j_end; j0 += kWarps * 4 * kUnroll) {
    uint4 kv[kUnroll], vv[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int j = j0 + u * 4 + sub;
      kv[u] = j < j_end ? *reinterpret_cast<const uint4 *>(kbase + int64_t(j) * HD + l8 * 8) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int j = j0 + u * 4 + sub;
      vv[u] = j < j_end ? *reinterpret_cast<const uint4 *>(vbase + int64_t(j) * HD + l8 * 8) : make_uint4(0, 0, 0, 0);
    }
    float sc[kUnroll][REP];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int j = j0 + u * 4 + sub;
      const __half *kh = reinterpret_cast<const __half *>(&kv[u]);
#pragma unroll
      for (int r = 0; r < REP; ++r) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) d = fmaf(qv[r][e], __half2float(kh[e]), d);
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        d += __shfl_xor_sync(0xffffffffu, d, 2);
        d += __shfl_xor_sync(0xffffffffu, d, 4);
        sc[u][r] = j < j_end ? __half2float(__float2half_rn(__half2float(__float2half_rn(d)) * scale)) : -INFINITY;
      }
    }
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      float mx = m[r];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) mx = fmaxf(mx, sc[u][r]);
      if (mx == -INFINITY) continue;           // no valid row in this step for this group
      const float c = softmax_weight(m[r], mx);
      l[r] *= c;
#pragma unroll
      for (int e = 0; e < 8; ++e) a[r][e] *= c;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const float pj = softmax_weight(sc[u][r], mx);
        l[r] += pj;
        const __half *vh = reinterpret_cast<const __half *>(&vv[u]);
#pragma unroll
        for (int e = 0; e < 8; ++e) a[r][e] = fmaf(pj, __half2float(vh[e]), a[r][e]);
      }
      m[r] = mx;
    }
  }
  // ---- merge: the 4 row groups of the warp, then the warps, then the splits ----------
#pragma unroll
  for (int r = 0; r < REP; ++r) {
#pragma unroll
    for (int o = 8; o <= 16; o <<= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[r], o);
      const float lo = __shfl_xor_sync(0xffffffffu, l[r], o);
      const float mn = fmaxf(m[r], mo);
      const float ws = softmax_weight(m[r], mn), wo = softmax_weight(mo, mn);
      l[r] = l[r] * ws + lo * wo;
#pragma unroll
      for (int e = 0; e < 8; ++e) a[r][e] = a[r][e] * ws + __shfl_xor_sync(0xffffffffu, a[r][e], o) * wo;
      m[r] = mn;
    }
  }
  if (sub == 0) {
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      if (l8 == 0) {
        red[warp][r][0] = m[r];
        red[warp][r][1] = l[r];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) red[warp][r][2 + l8 * 8 + e] = a[r][e];
    }
  }
  __syncthreads();
  float *mine = splits > 1 ? sp.part + (int64_t(bg) * splits + split) * REP * ST : nullptr;
  for (int i = threadIdx.x; i < REP * HD; i += blockDim.x) {
    const int r = i / HD, d = i % HD;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, red[w][r][0]);
    float lt = 0.f, at = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float wt = softmax_weight(red[w][r][0], mx);
      lt += red[w][r][1] * wt;
      at += red[w][r][2 + d] * wt;
    }
    if (splits == 1) {
      out[int64_t(b) * heads * HD + (g * REP + r) * HD + d] = __float2half_rn(at / lt);
    } else {
      if (d == 0) {
        mine[r * ST] = mx;
        mine[r * ST + 1] = lt;
      }
      mine[r * ST + 2 + d] = at;
    }
  }
  if (splits == 1) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(sp.counters + bg, 1) == splits - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float *all = sp.part + int64_t(bg) * splits * REP * ST;
  for (int i = threadIdx.x; i < REP * HD; i += blockDim.x) {
    const int r = i / HD, d = i % HD;
    float mx = -INFINITY;
    for (int s2 = 0; s2 < splits; ++s2) mx = fmaxf(mx, __ldcg(all + (s2 * REP + r) * ST));
    float lt = 0.f, at = 0.f;
    for (int s2 = 0; s2 < splits; ++s2) {
      const float *st = all + (s2 * REP + r) * ST;
      const float wt = softmax_weight(__ldcg(st), mx);
      lt += __ldcg(st + 1) * wt;
      at += __ldcg(st + 2 + d) * wt;
    }
    out[int64_t(b) * heads * HD + (g * REP + r) * HD + d] = __float2half_rn(at / lt);
  }
  if (threadIdx.x == 0) sp.counters[bg] = 0;   // ready for the next call
}

// h = half(half(silu(float(gate))) * up)  (torch_npu_smollm.py:189-190)
__global__ void silu_mul_kernel(const __half *__restrict__ gate, const __half *__restrict__ up, int in_stride,
                                __half *__restrict__ out, int rows, int cols) {
  pdl_launch();
  pdl_wait();
  const int64_t total = int64_t(rows) * cols;
  for (int64_t id = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; id < total; id += int64_t(gridDim.x) * blockDim.x) {
    const int r = int(id / cols), c = int(id % cols);
    const float gv = __half2float(gate[int64_t(r) * in_stride + c]);
    const __half act = __float2half_rn(__fdiv_rn(gv, 1.f + expf(-gv)));
    out[id] = __hmul(act, up[int64_t(r) * in_stride + c]);
  }
}

// A row producer fused with the correction projection of the linear that consumes it:
// CTA (row, j) builds the produced fp16 row in shared memory -- RMSNorm with the optional
// residual add (MODE 0, same staging as rmsnorm_kernel) or half(half(silu(g)) * u)
// (MODE 1, as silu_mul_kernel) -- the j == 0 CTA stores it (and the new hidden state),
// and every CTA computes z[row, 8j + w] = half(sum_k row_k V[8j + w, k]) for its 8 columns,
// one per warp (zero past the rank): the projection the GEMV epilogue then applies.
struct RowProjParams {
  const __half *x, *res;   // MODE 0: x, residual (or null); MODE 1: gate, up
  __half *res_out;         // MODE 0: half(x + residual), or null
  const __half *gamma;     // MODE 0
  __half *out;             // produced row [rows, dim]
  int dim, in_stride;      // MODE 1: gate / up row stride
  float eps;
  const __half *v;         // [rank, dim] or null
  int rank, zs;            // z row stride (rank rounded up to 32)
  __half *z;               // [rows, zs]
};

template <int MODE>
__global__ void __launch_bounds__(256) row_project_kernel(const RowProjParams p) {
  extern __shared__ __align__(16) __half rowbuf[];   // [dim]
  __shared__ float sh[32];
  pdl_launch();
  pdl_wait();
  const int64_t r = blockIdx.x;
  const bool store = blockIdx.y == 0;
  const int nvec = p.dim / 8;
  if constexpr (MODE == 0) {
    constexpr int MAXV = 8;
    float v[MAXV * 8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nvec) {
        uint4 a = *reinterpret_cast<const uint4 *>(p.x + r * p.dim + c * 8);
        const __half *ah = reinterpret_cast<const __half *>(&a);
        if (p.res) {
          uint4 b = *reinterpret_cast<const uint4 *>(p.res + r * p.dim + c * 8);
          const __half *bh = reinterpret_cast<const __half *>(&b);
          uint4 h;
          __half *hh = reinterpret_cast<__half *>(&h);
#pragma unroll
          for (int j = 0; j < 8; ++j) hh[j] = __float2half_rn(__half2float(ah[j]) + __half2float(bh[j]));
          if (p.res_out && store) *reinterpret_cast<uint4 *>(p.res_out + r * p.dim + c * 8) = h;
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i * 8 + j] = __half2float(hh[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i * 8 + j] = __half2float(ah[j]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(v[i * 8 + j], v[i * 8 + j], ss);
      }
    }
    const float total = block_sum(ss, sh);
    const float inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(total, float(p.dim)), p.eps));
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nvec) {
        uint4 g = *reinterpret_cast<const uint4 *>(p.gamma + c * 8);
        const __half *gh = reinterpret_cast<const __half *>(&g);
        uint4 o;
        __half *oh = reinterpret_cast<__half *>(&o);
#pragma unroll
        for (int j = 0; j < 8; ++j) oh[j] = __hmul(__float2half_rn(__fmul_rn(v[i * 8 + j], inv)), gh[j]);
        reinterpret_cast<uint4 *>(rowbuf)[c] = o;
        if (store) *reinterpret_cast<uint4 *>(p.out + r * p.dim + c * 8) = o;
      }
    }
  } else {
    for (int c = threadIdx.x; c < nvec; c += blockDim.x) {
      const uint4 g = *reinterpret_cast<const uint4 *>(p.x + r * p.in_stride + c * 8);
      const uint4 u = *reinterpret_cast<const uint4 *>(p.res + r * p.in_stride + c * 8);
      const __half *gh = reinterpret_cast<const __half *>(&g), *uh = reinterpret_cast<const __half *>(&u);
      uint4 o;
      __half *oh = reinterpret_cast<__half *>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float gv = __half2float(gh[j]);
        oh[j] = __hmul(__float2half_rn(__fdiv_rn(gv, 1.f + expf(-gv))), uh[j]);
      }
      reinterpret_cast<uint4 *>(rowbuf)[c] = o;
      if (store) *reinterpret_cast<uint4 *>(p.out + r * p.dim + c * 8) = o;
    }
  }
  if (!p.v) return;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int col = blockIdx.y * 8 + warp;
  float acc = 0.f;
  if (col < p.rank) {
    const __half *vr = p.v + int64_t(col) * p.dim;
#pragma unroll 4
    for (int c = lane; c < nvec; c += 32) {
      const uint4 a = reinterpret_cast<const uint4 *>(rowbuf)[c];
      const uint4 b = *reinterpret_cast<const uint4 *>(vr + c * 8);
      fma2_f16_f32(acc, a.x, b.x);
      fma2_f16_f32(acc, a.y, b.y);
      fma2_f16_f32(acc, a.z, b.z);
      fma2_f16_f32(acc, a.w, b.w);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0 && col < p.zs) p.z[r * p.zs + col] = __float2half_rn(col < p.rank ? acc : 0.f);
}

__global__ void add_kernel(const __half *__restrict__ a, const __half *__restrict__ b, __half *__restrict__ out,
                           int64_t count) {
  pdl_launch();
  pdl_wait();
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += int64_t(gridDim.x) * blockDim.x)
    out[i] = __float2half_rn(__half2float(a[i]) + __half2float(b[i]));
}

// Embedding rows (torch_npu_smollm_io.py:45-50).  Out-of-range ids yield zero rows.
__global__ void embed_kernel(const int64_t *__restrict__ ids, const __half *__restrict__ table,
                             __half *__restrict__ out, int64_t tokens, int dim, int64_t vocab) {
  pdl_launch();
  pdl_wait();
  const int64_t total = tokens * dim;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = i / dim;
    const int c = int(i % dim);
    const int64_t id = ids[t];
    out[i] = (id >= 0 && id < vocab) ? table[id * dim + c] : __float2half(0.f);
  }
}

// Greedy argmax per row, first index on ties (torch.argmax).
__global__ void __launch_bounds__(1024) argmax_kernel(const __half *__restrict__ logits, int vocab,
                                                      int64_t *__restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_launch();
  pdl_wait();
  const int64_t r = blockIdx.x;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const __half *row = logits + r * vocab;
  if ((vocab & 7) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    // 16-byte loads, every one in flight before the comparisons (ascending index within a
    // thread, so ties keep the first index)
    for (int c = threadIdx.x; c < vocab / 8; c += blockDim.x) {
      const uint4 q = *reinterpret_cast<const uint4 *>(row + 8 * c);
      const __half *h = reinterpret_cast<const __half *>(&q);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float v = __half2float(h[e]);
        if (v > best) { best = v; bi = 8 * c + e; }
      }
    }
  } else {
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
      const float v = __half2float(row[i]);
      if (v > best || (v == best && i < bi)) { best = v; bi = i; }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { sv[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < int(blockDim.x >> 5); ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) { best = sv[w]; bi = si[w]; }
    out[r] = bi == 0x7fffffff ? 0 : bi;
  }
}

}  // namespace lowbit

namespace lowbit_host {
using namespace lowbit;

static unsigned grid_1d(int64_t work, int block) {
  int64_t g = (work + block - 1) / block;
  if (g > 148 * 16) g = 148 * 16;
  return unsigned(g < 1 ? 1 : g);
}

cudaError_t launch_rmsnorm(const uint16_t *x, const uint16_t *res, uint16_t *res_out, const uint16_t *gamma,
                           uint16_t *out, int rows, int dim, float eps, cudaStream_t st) {
  int threads = 256;
  while (threads > 32 && (dim / 8) <= threads / 2) threads /= 2;
  return launch_k(rmsnorm_kernel, dim3(rows), dim3(threads), 0, st, reinterpret_cast<const __half *>(x),
                  reinterpret_cast<const __half *>(res), reinterpret_cast<__half *>(res_out),
                  reinterpret_cast<const __half *>(gamma), reinterpret_cast<__half *>(out), dim, eps);
}

// mode 0: RMSNorm (+ residual) rows, mode 1: SiLU-mul rows; z for the following linear.
cudaError_t launch_row_project(int mode, const uint16_t *x, const uint16_t *res, uint16_t *res_out,
                               const uint16_t *gamma, uint16_t *out, int rows, int dim, int in_stride, float eps,
                               const uint16_t *v, int rank, uint16_t *z, cudaStream_t st) {
  RowProjParams p;
  p.x = reinterpret_cast<const __half *>(x);
  p.res = reinterpret_cast<const __half *>(res);
  p.res_out = reinterpret_cast<__half *>(res_out);
  p.gamma = reinterpret_cast<const __half *>(gamma);
  p.out = reinterpret_cast<__half *>(out);
  p.dim = dim;
  p.in_stride = in_stride;
  p.eps = eps;
  p.v = reinterpret_cast<const __half *>(v);
  p.rank = v ? rank : 0;
  p.zs = v ? (rank + 31) / 32 * 32 : 32;
  p.z = reinterpret_cast<__half *>(z);
  const dim3 grid(rows, v ? p.zs / 8 : 1);   // 8 z columns (one per warp) per CTA
  const size_t smem = size_t(dim) * 2;
  if (mode == 0) {
    auto kern = row_project_kernel<0>;
    cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void *>(kern), int(smem));
    if (e != cudaSuccess) return e;
    return launch_k(kern, grid, dim3(256), smem, st, p);
  }
  auto kern = row_project_kernel<1>;
  cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void *>(kern), int(smem));
  if (e != cudaSuccess) return e;
  return launch_k(kern, grid, dim3(256), smem, st, p);
}

cudaError_t launch_rope(uint16_t *q, uint16_t *k, const int32_t *pos, const uint16_t *cos_t, const uint16_t *sin_t,
                        int table_rows, int tokens, int heads, int kvh, int hd, int q_stride, int k_stride,
                        cudaStream_t st) {
  const int64_t work = int64_t(tokens) * (heads + kvh) * (hd / 2);
  return launch_k(rope_kernel, dim3(grid_1d(work, 256)), dim3(256), 0, st, reinterpret_cast<__half *>(q),
                  reinterpret_cast<__half *>(k), pos, reinterpret_cast<const __half *>(cos_t),
                  reinterpret_cast<const __half *>(sin_t), table_rows, tokens, heads, kvh, hd, q_stride, k_stride);
}

cudaError_t launch_kv_append(const uint16_t *k, const uint16_t *v, int kv_stride, uint16_t *kc, uint16_t *vc,
                             const int32_t *lengths, int batch, int kvh, int hd, int max_pos, cudaStream_t st) {
  const int64_t work = int64_t(batch) * kvh * hd;
  return launch_k(kv_append_kernel, dim3(grid_1d(work, 256)), dim3(256), 0, st, reinterpret_cast<const __half *>(k),
                  reinterpret_cast<const __half *>(v), kv_stride, reinterpret_cast<__half *>(kc),
                  reinterpret_cast<__half *>(vc), lengths, batch, kvh, hd, max_pos);
}

// Position splits per (sequence, kv head): enough CTAs for ~3 per SM, at least 256
// positions per split, at most kMaxAttnSplits; none when the caller's workspace is too
// small or the arrival counters would not fit.  LOWBIT_ATTN_SPLITS forces a count (tuning).
constexpr int kMaxAttnSplits = 16;
constexpr int kAttnCounters = 4094;   // the workspace's GEMV arrival counters, minus two reserved

size_t attention_scratch_bytes(int batch, int heads, int splits) {
  return size_t(batch) * heads * splits * (2 + 64) * sizeof(float);
}

int attention_splits(int batch, int kvh, int heads, int max_pos, size_t scratch_bytes) {
  const int ctas = batch * kvh;
  int s = std::min((444 + ctas - 1) / ctas, std::max(1, max_pos / 256));
  if (const char *env = getenv("LOWBIT_ATTN_SPLITS")) s = atoi(env);
  s = std::max(1, std::min(s, kMaxAttnSplits));
  if (ctas > kAttnCounters) return 1;
  while (s > 1 && attention_scratch_bytes(batch, heads, s) > scratch_bytes) --s;
  return s;
}

template <int REP>
static cudaError_t launch_attention_rep(const uint16_t *q, int q_stride, uint16_t *kc, uint16_t *vc,
                                        const int32_t *lengths, uint16_t *out, int batch, int heads, int kvh,
                                        int max_pos, float scale, const RopeAppend &ra, int splits,
                                        const AttnSplit &sp, cudaStream_t st) {
  return launch_k(attention_decode_kernel<64, REP>, dim3(batch * kvh, splits), dim3(256), 0, st,
                  reinterpret_cast<const __half *>(q), q_stride, reinterpret_cast<__half *>(kc),
                  reinterpret_cast<__half *>(vc), lengths, reinterpret_cast<__half *>(out), heads, kvh, max_pos, scale,
                  ra, sp);
}

// counters: the workspace's arrival counters; scratch / scratch_bytes: the rest of it.
static cudaError_t launch_attention(const uint16_t *q, int q_stride, uint16_t *kc, uint16_t *vc,
                                    const int32_t *lengths, uint16_t *out, int batch, int heads, int kvh, int hd,
                                    int max_pos, float scale, const RopeAppend &ra, int *counters, void *scratch,
                                    size_t scratch_bytes, cudaStream_t st) {
  if (hd != 64) return cudaErrorInvalidValue;
  const int splits = counters && scratch ? attention_splits(batch, kvh, heads, max_pos, scratch_bytes) : 1;
  AttnSplit sp;
  sp.part = static_cast<float *>(scratch);
  sp.counters = counters;
  switch (heads / kvh) {
#define LB_ATTN_CASE(R) \
    case R: return launch_attention_rep<R>(q, q_stride, kc, vc, lengths, out, batch, heads, kvh, max_pos, scale, ra, splits, sp, st);
    LB_ATTN_CASE(1) LB_ATTN_CASE(2) LB_ATTN_CASE(3) LB_ATTN_CASE(4)
    LB_ATTN_CASE(5) LB_ATTN_CASE(6) LB_ATTN_CASE(7) LB_ATTN_CASE(8)
#undef LB_ATTN_CASE
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_attention_decode(const uint16_t *q, int q_stride, const uint16_t *kc, const uint16_t *vc,
                                    const int32_t *lengths, uint16_t *out, int batch, int heads, int kvh, int hd,
                                    int max_pos, float scale, int *counters, void *scratch, size_t scratch_bytes,
                                    cudaStream_t st) {
  // without the prologue nothing writes the caches
  return launch_attention(q, q_stride, const_cast<uint16_t *>(kc), const_cast<uint16_t *>(vc), lengths, out, batch,
                          heads, kvh, hd, max_pos, scale, RopeAppend{}, counters, scratch, scratch_bytes, st);
}

cudaError_t launch_attention_decode_rope(const uint16_t *q, int q_stride, const uint16_t *k_new, const uint16_t *v_new,
                                         int kv_stride, const uint16_t *cos_t, const uint16_t *sin_t, int table_rows,
                                         uint16_t *kc, uint16_t *vc, const int32_t *lengths, uint16_t *out, int batch,
                                         int heads, int kvh, int hd, int max_pos, float scale, int *counters,
                                         void *scratch, size_t scratch_bytes, cudaStream_t st) {
  RopeAppend ra;
  ra.k_new = reinterpret_cast<const __half *>(k_new);
  ra.v_new = reinterpret_cast<const __half *>(v_new);
  ra.kv_stride = kv_stride;
  ra.cos_t = reinterpret_cast<const __half *>(cos_t);
  ra.sin_t = reinterpret_cast<const __half *>(sin_t);
  ra.table_rows = table_rows;
  return launch_attention(q, q_stride, kc, vc, lengths, out, batch, heads, kvh, hd, max_pos, scale, ra, counters,
                          scratch, scratch_bytes, st);
}

cudaError_t launch_silu_mul(const uint16_t *gate, const uint16_t *up, int in_stride, uint16_t *out, int rows, int cols,
                            cudaStream_t st) {
  return launch_k(silu_mul_kernel, dim3(grid_1d(int64_t(rows) * cols, 256)), dim3(256), 0, st,
                  reinterpret_cast<const __half *>(gate), reinterpret_cast<const __half *>(up), in_stride,
                  reinterpret_cast<__half *>(out), rows, cols);
}

cudaError_t launch_add(const uint16_t *a, const uint16_t *b, uint16_t *out, int64_t count, cudaStream_t st) {
  return launch_k(add_kernel, dim3(grid_1d(count, 256)), dim3(256), 0, st, reinterpret_cast<const __half *>(a),
                  reinterpret_cast<const __half *>(b), reinterpret_cast<__half *>(out), count);
}

cudaError_t launch_embed(const int64_t *ids, const uint16_t *table, uint16_t *out, int64_t tokens, int dim,
                         int64_t vocab, cudaStream_t st) {
  return launch_k(embed_kernel, dim3(grid_1d(tokens * dim, 256)), dim3(256), 0, st, ids,
                  reinterpret_cast<const __half *>(table), reinterpret_cast<__half *>(out), tokens, dim, vocab);
}

cudaError_t launch_argmax(const uint16_t *logits, int rows, int vocab, int64_t *out, cudaStream_t st) {
  return launch_k(argmax_kernel, dim3(rows), dim3(1024), 0, st, reinterpret_cast<const __half *>(logits), vocab, out);
}

}  // namespace lowbit_host
