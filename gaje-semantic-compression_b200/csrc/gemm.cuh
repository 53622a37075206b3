// gemm.cuh -- Q4_0 matrix times a few activation vectors: the batched-decode
// projections (gaje_cuda_forward_batch) and the op-level M > 1 path of
// gaje_cuda_q4_0_gemv (the isolated GEMV sweep at M = 8).
//
// y[m][n] = flush(sum_b scale_b*A_b + min_b*X_b) + bias[n] with
// A_b = sum_k q_k x_mk over block b (the AVX2 arm of genomic.rs:267-336
// factored, as in the decode kernels).  A warp owns row pairs, a lane one
// 32-weight block of each; the lane turns each 8-nibble word of both rows into
// exact floats once and applies them to all MT activation vectors (held in
// shared memory, swizzled, with per-block sums), so the nibble work is shared
// by the vectors.  K is cut into splits of kSkChunk (grid.z): one split per
// CTA, and with more than one the CTA writes partial dots and the last CTA of
// the row tile adds the splits in order and runs the epilogue.
#pragma once

#include "megakernel.cuh"

namespace gaje {

constexpr int kSkThreads = 128;
constexpr int kSkWarps = kSkThreads / 32;
constexpr int kSkChunk = 1024;  // activations per vector per split (32 blocks)

__host__ __device__ inline size_t skinny_smem_bytes(int mt) {
  return size_t(mt) * (kSkChunk + kSkChunk / 32) * 4;
}

// The plain epilogue: y[m][row] = v.
struct EpiStore {
  float* y;
  int N;
  __device__ __forceinline__ void operator()(int m, int r, float v0, bool has1, float v1) const {
    y[(size_t)m * N + r] = v0;
    if (has1) y[(size_t)m * N + r + 1] = v1;
  }
};

// Optional RMSNorm of the activation rows while staging (see the kernel).
struct SkNorm {
  const float* w = nullptr;  // NORM: [K] norm weights
  float eps = 0.f;
  DevState* st = nullptr;    // NaN guards (NORM only), or nullptr
  const unsigned* pos = nullptr;
  int layer = 0;
};

// Work split: row pairs per warp, and for gridDim.z > 1 the split partials
// part[z][m][n] and one arrival counter per (x, y) tile (zero between
// launches; the last CTA resets its counter).
struct SkSplit {
  int ppw = 1;
  float* part = nullptr;
  unsigned* cnt = nullptr;
};

// One word (8 nibbles) of a row as four exact float pairs (q_{2i}, q_{2i+1}):
// each nibble is OR-ed into the mantissa of 2^23 at its own bit position p
// (bits p..p+3 of the word, or of the word >> 12 for the top three), then
// f * 2^-p - 2^(23-p) = q exactly in one packed FMA.
__device__ __forceinline__ void q4_word_pairs(uint32_t a, unsigned long long (&q)[4]) {
  const uint32_t M = 0x4B000000u, t = a >> 12;
  const float f0 = __uint_as_float((a & 0xFu) | M), f1 = __uint_as_float((a & 0xF0u) | M);
  const float f2 = __uint_as_float((a & 0xF00u) | M), f3 = __uint_as_float((a & 0xF000u) | M);
  const float f4 = __uint_as_float((a & 0xF0000u) | M), f5 = __uint_as_float((t & 0xF00u) | M);
  const float f6 = __uint_as_float((t & 0xF000u) | M), f7 = __uint_as_float((t & 0xF0000u) | M);
  // bit positions 0,4 | 8,12 | 16,8 | 12,16
  q[0] = ffma2(pack2(f0, f1), pack2(1.0f, 0.0625f), pack2(-8388608.0f, -524288.0f));
  q[1] = ffma2(pack2(f2, f3), pack2(0.00390625f, 0.000244140625f), pack2(-32768.0f, -2048.0f));
  q[2] = ffma2(pack2(f4, f5), pack2(1.52587890625e-05f, 0.00390625f), pack2(-128.0f, -32768.0f));
  q[3] = ffma2(pack2(f6, f7), pack2(0.000244140625f, 1.52587890625e-05f), pack2(-2048.0f, -128.0f));
}

// epi(m, r0, v0, has1, v1) receives rows r0 (and r0 + 1) of vector m, flushed
// and with the bias added.
//
// With NORM, the staged activations are RMSNorm(x) = (x * inv) * norm_w with
// inv = 1/sqrt(sum(x^2)/K + eps) per vector (norm.rs:17-87), computed by each
// CTA for its MT vectors (K = d for the projections that follow a norm) in
// the same pass that stages the raw values, then applied in shared memory;
// with `st`, the CTAs of column 0 also raise the block-input and
// normed-output NaN guards of block/forward.rs:11-13 and :22-24 at each
// vector's position.
//
// Launch: grid (ceil(N / (2 * kSkWarps * ppw)), ceil(M/MT), Z), kSkThreads,
// skinny_smem_bytes(MT); x rows 16-byte aligned (K % 32 == 0).  Z = 1: the
// CTA walks all K splits itself (sums kept per lane in shared memory); Z =
// ceil(K/kSkChunk): one split per CTA through sp.part / sp.cnt.  The next
// item's weight words are always fetched before the current one is computed
// (the first ones before griddepcontrol.wait: weights never depend on the
// previous kernel).
template <int MT, bool NORM, class Epi>
__global__ void __launch_bounds__(kSkThreads) k_q4_gemm_skinny(Q4View W, const float* x, int M, SkNorm nm, SkSplit sp,
                                                               Epi epi) {
  static_assert(MT == 8, "the 16-value lane reduction assumes 8 vectors x 2 rows");
  constexpr int kMaxPpw = 8;
  extern __shared__ __align__(16) float sk_smem[];
  __shared__ float inv_s[MT];
  __shared__ float red[kSkWarps * kMaxPpw * MT * 2];  // per-lane sums over splits (Z = 1); row sums of squares
  __shared__ int is_last;
  __shared__ unsigned bad_s;
  float* xs = sk_smem;                    // [MT][kSkChunk]
  float* xsum = sk_smem + MT * kSkChunk;  // [MT][kSkChunk / 32]
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int m0 = blockIdx.y * MT;
  const int mt = min(MT, M - m0);
  const int nbt = W.K >> 5;
  const int nsplit = (W.K + kSkChunk - 1) / kSkChunk;
  const bool gsplit = gridDim.z > 1;
  const int zb = gsplit ? (int)blockIdx.z : 0, ze = gsplit ? zb + 1 : nsplit;
  const bool multi = !gsplit && nsplit > 1;
  const int ppw = sp.ppw;
  const int pair0 = (blockIdx.x * kSkWarps + wid) * ppw;
  auto fetch = [&](int z, int i, uint4& qa, uint4& qb, uint32_t& sa, uint32_t& sb) {
    const int r = 2 * (pair0 + i), b = z * 32 + lane;
    qa = qb = make_uint4(0u, 0u, 0u, 0u);
    sa = sb = 0u;
    if (z < ze && b < nbt && r < W.N) {
      qa = __ldg(W.qs + (size_t)r * W.nb + b);
      sa = __ldg(W.sm + (size_t)r * W.nbp + b);
      if (r + 1 < W.N) {
        qb = __ldg(W.qs + (size_t)(r + 1) * W.nb + b);
        sb = __ldg(W.sm + (size_t)(r + 1) * W.nbp + b);
      }
    }
  };
  uint4 qa, qb;
  uint32_t sa, sb;
  fetch(zb, 0, qa, qb, sa, sb);
  pdl_wait();
  pdl_trigger();
  const float4* x4 = reinterpret_cast<const float4*>(xs + (lane << 5));
  const int sw = lane & 7;
  const int m = lane >> 2;  // the vector whose two rows this lane holds after the reduction
  const bool guard = NORM && nm.st && blockIdx.x == 0;
  if (tid == 0) bad_s = 0u;
  for (int z = zb; z < ze; ++z) {
    const int k0 = z * kSkChunk;
    const int kc = min(kSkChunk, W.K - k0);  // a multiple of 32
    const int nf4 = kc >> 2;                  // float4s of a vector in this split (a multiple of 8)
    const bool lane_on = lane < (kc >> 5);
    __syncthreads();  // the previous split's activations are consumed
    // pass 1: this split's raw activations -> xs (swizzled by block).  With
    // NORM, the first pass reads whole rows: their sums of squares and NaN
    // scan (the parts outside this split are read for the sums only).
    {
      const bool whole = NORM && z == zb;
      const int n4 = whole ? (W.K >> 2) : nf4;
      const int fbase = whole ? (k0 >> 2) : 0;  // this split's first float4 in the loop's index space
      float ssp[MT];
#pragma unroll
      for (int j = 0; j < MT; ++j) ssp[j] = 0.f;
      unsigned badm = 0u;
      for (int f0 = 0; f0 < n4; f0 += kSkThreads) {
        const int f = f0 + tid;
        const bool in = f < n4;
        const float* src = x + (whole ? 0 : k0);
        float4 v[MT];
#pragma unroll
        for (int j = 0; j < MT; ++j)
          v[j] = (in && j < mt) ? __ldg(reinterpret_cast<const float4*>(src + (size_t)(m0 + j) * W.K) + f)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        const int fs = f - fbase;
        const bool mine = in && fs >= 0 && fs < nf4;
        const int blk = fs >> 3, c = fs & 7;
#pragma unroll
        for (int j = 0; j < MT; ++j) {
          if (whole) {
            ssp[j] = fmaf(v[j].x, v[j].x, ssp[j]);
            ssp[j] = fmaf(v[j].y, v[j].y, ssp[j]);
            ssp[j] = fmaf(v[j].z, v[j].z, ssp[j]);
            ssp[j] = fmaf(v[j].w, v[j].w, ssp[j]);
            if ((v[j].x != v[j].x) | (v[j].y != v[j].y) | (v[j].z != v[j].z) | (v[j].w != v[j].w)) badm |= 1u << j;
          }
          if (mine) reinterpret_cast<float4*>(xs + j * kSkChunk)[blk * 8 + (c ^ (blk & 7))] = v[j];
        }
      }
      if (whole) {
#pragma unroll
        for (int j = 0; j < MT; ++j) {
          const float t = warp_sum(ssp[j]);
          if (lane == 0) red[wid * MT + j] = t;
        }
        if (guard && badm) atomicOr(&bad_s, badm);
      }
    }
    __syncthreads();
    if (NORM && z == zb) {
      if (tid < MT) {
        float t = 0.f;
        for (int w = 0; w < kSkWarps; ++w) t += red[w * MT + tid];
        inv_s[tid] = 1.0f / sqrtf(t / (float)W.K + nm.eps);
        if (guard && blockIdx.z == 0 && tid < mt && (bad_s >> tid) & 1u)
          nan_flag(nm.st, nm.pos[m0 + tid], nm.layer, kNanInput);
      }
      __syncthreads();
    }
    // pass 2 (shared memory only): NORM -> (x * inv) * w in place (the
    // reference's order); the block sums -> xsum
    {
      unsigned badn = 0u;
      for (int f0 = 0; f0 < nf4; f0 += kSkThreads) {
        const int f = f0 + tid;
        const bool in = f < nf4;
        const int blk = f >> 3, c = f & 7;
        float4* slot0 = reinterpret_cast<float4*>(xs) + blk * 8 + (c ^ (blk & 7));
        float4 nw = make_float4(1.f, 1.f, 1.f, 1.f);
        if (NORM && in) nw = __ldg(reinterpret_cast<const float4*>(nm.w + k0) + f);
#pragma unroll
        for (int j = 0; j < MT; ++j) {
          float4 u = in ? slot0[j * (kSkChunk / 4)] : make_float4(0.f, 0.f, 0.f, 0.f);
          if constexpr (NORM) {
            const float inv = inv_s[j];
            u.x = (u.x * inv) * nw.x;
            u.y = (u.y * inv) * nw.y;
            u.z = (u.z * inv) * nw.z;
            u.w = (u.w * inv) * nw.w;
            if (in) slot0[j * (kSkChunk / 4)] = u;
            if (guard && in && j < mt && ((u.x != u.x) | (u.y != u.y) | (u.z != u.z) | (u.w != u.w))) badn |= 1u << j;
          }
          float s = (u.x + u.y) + (u.z + u.w);
          s += __shfl_xor_sync(0xffffffffu, s, 1);
          s += __shfl_xor_sync(0xffffffffu, s, 2);
          s += __shfl_xor_sync(0xffffffffu, s, 4);
          if (in && c == 0) xsum[j * (kSkChunk / 32) + blk] = s;
        }
      }
      if (guard && badn)
        for (int j = 0; j < MT; ++j)
          if ((badn >> j) & 1u) nan_flag(nm.st, nm.pos[m0 + j], nm.layer, kNanAttnNorm);
    }
    __syncthreads();
    for (int i = 0; i < ppw; ++i) {
      uint4 nqa, nqb;
      uint32_t nsa, nsb;
      if (i + 1 < ppw) fetch(z, i + 1, nqa, nqb, nsa, nsb);
      else fetch(z + 1, 0, nqa, nqb, nsa, nsb);
      const int r0 = 2 * (pair0 + i);
      // v[2j + row]: this lane's block of row r0 + row against vector j
      float v[2 * MT];
#pragma unroll
      for (int k = 0; k < 2 * MT; ++k) v[k] = 0.f;
      if (lane_on && r0 < W.N) {
        unsigned long long acc[2 * MT];
#pragma unroll
        for (int k = 0; k < 2 * MT; ++k) acc[k] = 0ull;  // (+0.0f, +0.0f)
        const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w};
        const uint32_t wb[4] = {qb.x, qb.y, qb.z, qb.w};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          unsigned long long pa[4], pb[4];
          q4_word_pairs(wa[w], pa);
          q4_word_pairs(wb[w], pb);
#pragma unroll
          for (int j = 0; j < MT; ++j) {
            const float4 xa = x4[j * (kSkChunk / 4) + ((2 * w) ^ sw)];
            const float4 xb = x4[j * (kSkChunk / 4) + ((2 * w + 1) ^ sw)];
            const unsigned long long x01 = pack2(xa.x, xa.y), x23 = pack2(xa.z, xa.w);
            const unsigned long long x45 = pack2(xb.x, xb.y), x67 = pack2(xb.z, xb.w);
            acc[2 * j] = ffma2(pa[0], x01, acc[2 * j]);
            acc[2 * j] = ffma2(pa[1], x23, acc[2 * j]);
            acc[2 * j] = ffma2(pa[2], x45, acc[2 * j]);
            acc[2 * j] = ffma2(pa[3], x67, acc[2 * j]);
            acc[2 * j + 1] = ffma2(pb[0], x01, acc[2 * j + 1]);
            acc[2 * j + 1] = ffma2(pb[1], x23, acc[2 * j + 1]);
            acc[2 * j + 1] = ffma2(pb[2], x45, acc[2 * j + 1]);
            acc[2 * j + 1] = ffma2(pb[3], x67, acc[2 * j + 1]);
          }
        }
        float sc0, mn0, sc1, mn1;
        unpack_sm(sa, sc0, mn0);
        unpack_sm(sb, sc1, mn1);
#pragma unroll
        for (int j = 0; j < MT; ++j) {
          const float xbs = xsum[j * (kSkChunk / 32) + lane];
          float a0, a1, c0, c1;
          unpack2(acc[2 * j], a0, a1);
          unpack2(acc[2 * j + 1], c0, c1);
          v[2 * j] = fmaf(sc0, a0 + a1, mn0 * xbs);
          v[2 * j + 1] = fmaf(sc1, c0 + c1, mn1 * xbs);
        }
      }
      // 16 values over 32 lanes: lanes 2k and 2k+1 end with the sum of value k
#pragma unroll
      for (int o = 16, h = MT; o >= 2; o >>= 1, h >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int k = 0; k < h; ++k) {
          const float send = up ? v[k] : v[k + h];
          const float keep = up ? v[k + h] : v[k];
          v[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      const float tot = v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
      const float tot1 = __shfl_down_sync(0xffffffffu, tot, 2);  // row r0 + 1 of the same vector
      if ((lane & 3) == 0 && r0 < W.N && m < mt) {
        const bool has1 = r0 + 1 < W.N;
        if (gsplit) {
          float* pp = sp.part + ((size_t)z * M + m0 + m) * W.N + r0;
          pp[0] = tot;
          if (has1) pp[1] = tot1;
        } else if (multi) {  // the same lane adds every split of this (pair, vector), in order
          float* rr = red + ((wid * kMaxPpw + i) * MT + m) * 2;
          const float s0 = z == 0 ? tot : rr[0] + tot, s1 = z == 0 ? tot1 : rr[1] + tot1;
          if (z + 1 < ze) {
            rr[0] = s0;
            rr[1] = s1;
          } else {
            const float b0 = W.bias ? __ldg(W.bias + r0) : 0.f;
            const float b1 = (W.bias && has1) ? __ldg(W.bias + r0 + 1) : 0.f;
            epi(m0 + m, r0, flush_small(s0) + b0, has1, flush_small(s1) + b1);
          }
        } else {
          const float b0 = W.bias ? __ldg(W.bias + r0) : 0.f;
          const float b1 = (W.bias && has1) ? __ldg(W.bias + r0 + 1) : 0.f;
          epi(m0 + m, r0, flush_small(tot) + b0, has1, flush_small(tot1) + b1);
        }
      }
      qa = nqa;
      qb = nqb;
      sa = nsa;
      sb = nsb;
    }
  }
  if (!gsplit) return;
  // the last CTA of this row tile adds the splits in order and finishes
  __threadfence();
  __syncthreads();
  unsigned* cnt = sp.cnt + blockIdx.y * gridDim.x + blockIdx.x;
  if (tid == 0) is_last = (atomicAdd(cnt, 1u) == gridDim.z - 1u);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const int npairs = kSkWarps * ppw;
  for (int it = tid; it < npairs * MT; it += kSkThreads) {
    const int j = it / npairs, pr = it - j * npairs;
    const int r0 = 2 * (blockIdx.x * npairs + pr);
    if (j >= mt || r0 >= W.N) continue;
    const bool has1 = r0 + 1 < W.N;
    float s0 = 0.f, s1 = 0.f;
    for (int z = 0; z < (int)gridDim.z; ++z) {
      const float* pp = sp.part + ((size_t)z * M + m0 + j) * W.N + r0;
      s0 += __ldcg(pp);
      if (has1) s1 += __ldcg(pp + 1);
    }
    const float b0 = W.bias ? __ldg(W.bias + r0) : 0.f;
    const float b1 = (W.bias && has1) ? __ldg(W.bias + r0 + 1) : 0.f;
    epi(m0 + j, r0, flush_small(s0) + b0, has1, flush_small(s1) + b1);
  }
  if (tid == 0) *cnt = 0u;
}

}  // namespace gaje
