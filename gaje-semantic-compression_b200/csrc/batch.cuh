// batch.cuh -- one decode step for B independent streams of the same model
// (gaje_cuda_forward_batch; BASELINE configs[3] decode and the per-rank body
// of configs[4]).  Each stream has its own KV cache and position; the weights
// of a step are read once for all B streams.
//
// A step is a chain of kernels on the model's stream, captured once per batch
// size as a CUDA graph and chained with programmatic dependent launch: the
// embedding rows, then per block QKV (RMSNorm of the B residual rows while
// staging, Q4 GEMM for B vectors, RoPE at each stream's position, the k/v rows
// written straight into the stream's cache), split-K attention per (stream,
// KV head, split), O-proj + residual, gate/up (RMSNorm while staging) +
// SwiGLU, down + residual; then the output norm fused into the f32 lm_head
// for B vectors and a first-max argmax per stream.  Arithmetic per stream is
// the single-stream path's (the reference's forward_core,
// src/nn/llm/forward.rs:7-63): RMSNorm as (x*inv)*w (norm.rs:17-87), Q4 dots
// with the |t|<1e-6 flush then the bias (genomic.rs:331-335,
// linear/forward.rs:113-115), split RoPE / interleaved RoPE, the attention of
// attention.rs:88-127, swiglu_balanced.
#pragma once

#include "gemm.cuh"

namespace gaje {

// Per-step stream table (device arrays of B entries).
struct BatchStreams {
  const unsigned* tok;  // input token
  const unsigned* pos;  // position = the stream's cache length before the step
  const unsigned* sid;  // stream id (selects the KV cache)
};

// The batched KV caches: [stream][layer][nkv][max_ctx][hd] f32, K and V.
struct BatchCache {
  float* k;
  float* v;
  int L, nkv, max_ctx, hd;
  __host__ __device__ __forceinline__ size_t row(unsigned sid, int l, int g, unsigned pos) const {
    return ((((size_t)sid * L + l) * nkv + g) * max_ctx + pos) * hd;
  }
};

__global__ void k_embed_batch(const float* embd, int V, int d, BatchStreams bs, float* x) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const float* src = embd + (size_t)(bs.tok[b] % (unsigned)V) * d;  // get_row_core: row token % V
  for (int i = threadIdx.x; i < d; i += blockDim.x) x[(size_t)b * d + i] = __ldg(src + i);
}

// QKV epilogue: the unit u = r0/2 is a RoPE pair (rows stored pair-interleaved
// by the loader): q heads go to q[b], k rows (rotated) and v rows to the
// stream's cache at its position.
struct EpiQkvBatch {
  float* q;  // [B][nh*hd]
  BatchCache cache;
  BatchStreams bs;
  const float2* rope;  // [max_ctx][hd/2] (cos, sin)
  int nh, nkv, hd, rope_split, layer;
  __device__ __forceinline__ void operator()(int b, int r0, float y0, bool, float y1) const {
    const int half = hd >> 1;
    const int u = r0 >> 1;
    const int head = u / half, i = u - head * half;
    const int c0 = rope_split ? i : 2 * i;
    const int c1 = rope_split ? i + half : 2 * i + 1;
    const unsigned pos = bs.pos[b];
    if (head < nh + nkv) {  // RoPE: v0*cos - v1*sin, v0*sin + v1*cos
      const float2 cs = rope[(size_t)pos * half + i];
      const float o0 = y0 * cs.x - y1 * cs.y;
      const float o1 = y0 * cs.y + y1 * cs.x;
      y0 = o0;
      y1 = o1;
    }
    float* dst;
    if (head < nh) dst = q + (size_t)b * nh * hd + head * hd;
    else if (head < nh + nkv) dst = cache.k + cache.row(bs.sid[b], layer, head - nh, pos);
    else dst = cache.v + cache.row(bs.sid[b], layer, head - nh - nkv, pos);
    dst[c0] = y0;
    dst[c1] = y1;
  }
};

// x[b][row] += y (the residual adds of block/forward.rs:75-77, :132-136); for
// the down projection also the NaN guards of :128-130 and :138-140.
struct EpiResidBatch {
  float* x;
  int N;
  DevState* st;  // non-null: the down-projection guards
  BatchStreams bs;
  int layer;
  __device__ __forceinline__ void operator()(int b, int r, float y0, bool has1, float y1) const {
    for (int k = 0; k < 2; ++k) {
      if (k == 1 && !has1) break;
      const float y = k ? y1 : y0;
      float* xp = x + (size_t)b * N + r + k;
      const float xn = *xp + y;
      if (st) {
        if (y != y) nan_flag(st, bs.pos[b], layer, kNanProjFfn);
        if (xn != xn) nan_flag(st, bs.pos[b], layer, kNanResidual);
      }
      *xp = xn;
    }
  }
};

// gate/up pair (rows stored pair-interleaved) -> swiglu_balanced -> act[b][u].
struct EpiSwigluBatch {
  float* act;
  int ff;
  DevState* st;
  BatchStreams bs;
  int layer;
  __device__ __forceinline__ void operator()(int b, int r0, float g, bool, float u) const {
    if (u != u) nan_flag(st, bs.pos[b], layer, kNanUp);
    const float a = swiglu_balanced(g, u);
    if (a != a) nan_flag(st, bs.pos[b], layer, kNanFfnOut);
    act[(size_t)b * ff + (r0 >> 1)] = a;
  }
};

// Attention of stream blockIdx.z over its cache (the step's row is already in
// it): the single-stream split kernel's body with per-stream arguments.
struct AttnBatchArgs {
  const float* q;  // [B][nh*hd]
  float* out;      // [B][nh*hd]
  BatchCache cache;
  BatchStreams bs;
  float* part_o;   // [B][nkv][kAttnMaxSplits][G][hd]
  float* part_ml;  // [B][nkv][kAttnMaxSplits][G][2]
  unsigned* cnt;   // [B][nkv], zero between launches
  int layer, nh;
  float scale;
  int max_splits;  // splits per (stream, KV head) at most (the grid's y)
};
__global__ void __launch_bounds__(kAttnThreads) k_attn_batch(AttnBatchArgs B) {
  const int b = blockIdx.z;
  const int G = B.nh / B.cache.nkv, hd = B.cache.hd, nkv = B.cache.nkv;
  AttnArgs a{};
  a.q = B.q + (size_t)b * B.nh * hd;
  a.out = B.out + (size_t)b * B.nh * hd;
  a.kc = B.cache.k + B.cache.row(B.bs.sid[b], B.layer, 0, 0);
  a.vc = B.cache.v + B.cache.row(B.bs.sid[b], B.layer, 0, 0);
  a.part_o = B.part_o + (size_t)b * nkv * kAttnMaxSplits * G * hd;
  a.part_ml = B.part_ml + (size_t)b * nkv * kAttnMaxSplits * G * 2;
  a.cnt = B.cnt + (size_t)b * nkv;
  a.ctx = int(B.bs.pos[b]) + 1;
  a.stride = B.cache.max_ctx;
  a.nh = B.nh;
  a.nkv = nkv;
  a.hd = hd;
  a.scale = B.scale;
  a.st = nullptr;
  a.fresh = 1;  // the stream's row at pos is written by the QKV kernel just before
  a.max_splits = B.max_splits;
  attn_split(a, blockIdx.x, blockIdx.y);
}

// Causal attention for a prefill chunk of one stream: rows m = 0..n-1 at
// positions p0 + m, each attending to its stream's cached positions
// 0..p0+m (the chunk's own k/v rows are written by the QKV kernel before
// this one).  attention.rs:88-127 per (row, head): s_t = q.k_t * scale,
// softmax, out = sum p_t v_t with inv = 1/(sum + 1e-12); here as a
// flash-style pass over 64-position tiles with a running max and sum (the
// same values, another rounding order).  CTA: QB consecutive rows x the G
// query heads of one KV head, padded to 96 (row, head) pairs; K/V tiles in
// shared memory shared by all of them; 256 threads as a 16 x 16 grid, each
// holding a 6 x 4 block of scores and a 6-pair x (hd/64) float4 block of the
// output in registers, so every shared-memory load feeds several FMAs.
constexpr int kApThreads = 256;
constexpr int kApT = 64;   // key positions per tile
constexpr int kApQG = 96;  // (row, head) pairs per CTA, padded
__host__ __device__ inline int attn_prefill_qb(int G) {
  const int q = kApQG / G;
  return q < 1 ? 1 : q;
}
__host__ __device__ inline size_t attn_prefill_smem(int G, int hd) {
  return size_t(kApQG) * (hd + 4) * 4    // Qs (rows padded by 4 floats)
         + size_t(kApT) * (hd + 4) * 4   // Ks
         + size_t(kApT) * hd * 4         // Vs
         + size_t(kApQG) * (kApT + 4) * 4  // scores / probabilities
         + size_t(kApQG) * 3 * 4;        // running max, sum, rescale
}
struct AttnPrefillArgs {
  const float* q;   // [n][nh*hd]
  float* out;       // [n][nh*hd]
  const float* kc;  // this layer's cache of the stream: [nkv][max_ctx][hd]
  const float* vc;
  int n, p0, nh, nkv, hd, max_ctx;
  float scale;
};
__global__ void __launch_bounds__(kApThreads) k_attn_prefill(AttnPrefillArgs A) {
  extern __shared__ __align__(16) float ap_smem[];
  const int G = A.nh / A.nkv, hd = A.hd, hd4 = hd >> 2;
  const int QB = attn_prefill_qb(G), QG = QB * G;
  // the last row blocks (the longest causal spans) are scheduled first
  const int g = blockIdx.y, m0 = (gridDim.x - 1 - blockIdx.x) * QB;
  const int qs = hd + 4, ps = kApT + 4;      // padded row strides (floats)
  float* Qs = ap_smem;                       // [96][hd + 4]
  float* Ks = Qs + kApQG * qs;               // [64][hd + 4]
  float* Vs = Ks + kApT * qs;                // [64][hd]
  float* Ps = Vs + kApT * hd;                // [96][64 + 4]
  float* rmax = Ps + kApQG * ps;
  float* rsum = rmax + kApQG;
  float* ralpha = rsum + kApQG;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int ta = tid >> 4, tb = tid & 15;    // the thread's place in the 16 x 16 grid
  pdl_wait();
  pdl_trigger();
  const int last = min(A.n, m0 + QB) - 1;    // the CTA's last live row
  // pairs qh = (row i, head j): q of head g*G + j of row m0 + i; pads are zero
  for (int idx = tid; idx < kApQG * hd4; idx += kApThreads) {
    const int qh = idx / hd4, e4 = idx - qh * hd4;
    const int i = qh / G, j = qh - i * G;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (qh < QG && m0 + i <= last)
      v = __ldcg(reinterpret_cast<const float4*>(A.q + (size_t)(m0 + i) * A.nh * hd + (g * G + j) * hd) + e4);
    reinterpret_cast<float4*>(Qs + qh * qs)[e4] = v;
  }
  for (int qh = tid; qh < kApQG; qh += kApThreads) {
    rmax[qh] = -INFINITY;
    rsum[qh] = 0.f;
  }
  constexpr int kMaxD = 2;  // float4 columns of the output per thread: hd <= 128
  float4 o[6][kMaxD];
#pragma unroll
  for (int i = 0; i < 6; ++i)
#pragma unroll
    for (int k = 0; k < kMaxD; ++k) o[i][k] = make_float4(0.f, 0.f, 0.f, 0.f);
  const int maxpos = A.p0 + last;            // the farthest position any of its rows sees
  const float* kbase = A.kc + (size_t)g * A.max_ctx * hd;
  const float* vbase = A.vc + (size_t)g * A.max_ctx * hd;
  for (int t0 = 0; t0 <= maxpos; t0 += kApT) {
    __syncthreads();  // the previous tile is consumed
    for (int idx = tid; idx < kApT * hd4; idx += kApThreads) {
      const int j = idx / hd4, e4 = idx - j * hd4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (t0 + j <= maxpos) {
        kv = __ldcg(reinterpret_cast<const float4*>(kbase + (size_t)(t0 + j) * hd) + e4);
        vv = __ldcg(reinterpret_cast<const float4*>(vbase + (size_t)(t0 + j) * hd) + e4);
      }
      reinterpret_cast<float4*>(Ks + j * qs)[e4] = kv;
      reinterpret_cast<float4*>(Vs)[idx] = vv;
    }
    __syncthreads();
    // scores: pairs ta + 16r (r < 6) x positions tb + 16c (c < 4)
    {
      float acc[6][4];
#pragma unroll
      for (int r = 0; r < 6; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = 0.f;
      for (int e4 = 0; e4 < hd4; ++e4) {
        float4 kq[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) kq[c] = reinterpret_cast<const float4*>(Ks + (tb + 16 * c) * qs)[e4];
#pragma unroll
        for (int r = 0; r < 6; ++r) {
          const float4 a = reinterpret_cast<const float4*>(Qs + (ta + 16 * r) * qs)[e4];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            acc[r][c] = fmaf(a.x, kq[c].x, acc[r][c]);
            acc[r][c] = fmaf(a.y, kq[c].y, acc[r][c]);
            acc[r][c] = fmaf(a.z, kq[c].z, acc[r][c]);
            acc[r][c] = fmaf(a.w, kq[c].w, acc[r][c]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < 6; ++r) {
        const int qh = ta + 16 * r, i = qh / G;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int j = tb + 16 * c;
          const bool live = qh < QG && m0 + i <= last && t0 + j <= A.p0 + m0 + i;
          Ps[qh * ps + j] = live ? acc[r][c] * A.scale : -INFINITY;
        }
      }
    }
    __syncthreads();
    // running softmax per pair: a warp per pair, two positions per lane
    for (int qh = wid; qh < kApQG; qh += kApThreads / 32) {
      const float s0 = Ps[qh * ps + lane], s1 = Ps[qh * ps + lane + 32];
      const float mo = rmax[qh];
      const float mn = fmaxf(mo, warp_max(fmaxf(s0, s1)));
      float p0 = 0.f, p1 = 0.f, alpha = 1.f;
      if (mn > -INFINITY) {  // pads and rows past the chunk see nothing at all
        p0 = expf(s0 - mn);
        p1 = expf(s1 - mn);
        alpha = expf(mo - mn);
      }
      Ps[qh * ps + lane] = p0;
      Ps[qh * ps + lane + 32] = p1;
      const float psum = warp_sum(p0 + p1);
      if (lane == 0) {
        rsum[qh] = rsum[qh] * alpha + psum;
        rmax[qh] = mn;
        ralpha[qh] = alpha;
      }
    }
    __syncthreads();
    // O = O * alpha + P V: pairs ta + 16r x float4 columns tb + 16k
#pragma unroll
    for (int r = 0; r < 6; ++r) {
      const float al = ralpha[ta + 16 * r];
#pragma unroll
      for (int k = 0; k < kMaxD; ++k) {
        o[r][k].x *= al;
        o[r][k].y *= al;
        o[r][k].z *= al;
        o[r][k].w *= al;
      }
    }
    for (int j = 0; j < kApT; ++j) {
      float4 v[kMaxD];
#pragma unroll
      for (int k = 0; k < kMaxD; ++k)
        v[k] = (tb + 16 * k < hd4) ? reinterpret_cast<const float4*>(Vs + j * hd)[tb + 16 * k]
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < 6; ++r) {
        const float p = Ps[(ta + 16 * r) * ps + j];
#pragma unroll
        for (int k = 0; k < kMaxD; ++k) {
          o[r][k].x = fmaf(p, v[k].x, o[r][k].x);
          o[r][k].y = fmaf(p, v[k].y, o[r][k].y);
          o[r][k].z = fmaf(p, v[k].z, o[r][k].z);
          o[r][k].w = fmaf(p, v[k].w, o[r][k].w);
        }
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 6; ++r) {
    const int qh = ta + 16 * r, i = qh / G, j = qh - i * G;
    if (qh >= QG || m0 + i > last) continue;
    const float inv = 1.0f / (rsum[qh] + 1e-12f);
#pragma unroll
    for (int k = 0; k < kMaxD; ++k) {
      const int e4 = tb + 16 * k;
      if (e4 >= hd4) continue;
      const float4 v = make_float4(o[r][k].x * inv, o[r][k].y * inv, o[r][k].z * inv, o[r][k].w * inv);
      reinterpret_cast<float4*>(A.out + (size_t)(m0 + i) * A.nh * hd + (g * G + j) * hd)[e4] = v;
    }
  }
}

// Output RMSNorm + f32 lm_head for B vectors (llm/forward.rs:28,44-46,
// linear/forward.rs:20-32, no flush) + first-max argmax per stream
// (llm/forward.rs:262-271).  Every CTA normalises the B residual rows into
// shared memory ((x*inv)*w, norm.rs:17-87); a warp then takes RPW vocab rows
// at a time, so each activation float4 read from shared memory serves RPW
// rows, with RPW x 2 weight float4 loads in flight per lane; per-CTA best
// keys, and the last CTA reduces them.
constexpr int kLbThreads = 256;
struct LmBatchArgs {
  const float* W;       // [V][d]
  const float* bias;    // [V] or nullptr
  const float* x;       // [B][d] residual rows (before the output norm)
  const float* norm_w;  // [d]
  float eps;
  float* logits;        // [B][V]
  unsigned long long* part;  // [grid][B]
  unsigned* cnt;        // zero between launches
  unsigned* argmax;     // [B] first-max index (row_offset added), or nullptr
  unsigned long long* keys;  // [B] the winning amax_key of each vector, or nullptr
  unsigned row_offset;  // global index of W's row 0 (a vocab shard's first row)
  int V, d, B, rows_per_cta;
};
template <int MB, int RPW>
__global__ void __launch_bounds__(kLbThreads) k_lmhead_batch(LmBatchArgs A) {
  extern __shared__ __align__(16) float lb_smem[];
  __shared__ unsigned long long wbest[kLbThreads / 32][MB];
  __shared__ int is_last;
  constexpr int U = 2;  // float4 steps per row in flight
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = kLbThreads / 32;
  const int d = A.d, K4 = d >> 2;
  pdl_wait();
  pdl_trigger();
  for (int b = wid; b < A.B; b += nw) {  // warp b: RMSNorm of row b
    const float4* xr = reinterpret_cast<const float4*>(A.x + (size_t)b * d);
    float ss = 0.f;
    for (int j = lane; j < K4; j += 32) {
      const float4 v = __ldcg(xr + j);
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)d + A.eps);
    float4* o = reinterpret_cast<float4*>(lb_smem + (size_t)b * d);
    const float4* w = reinterpret_cast<const float4*>(A.norm_w);
    for (int j = lane; j < K4; j += 32) {
      const float4 v = __ldcg(xr + j), g = __ldg(w + j);
      o[j] = make_float4((v.x * inv) * g.x, (v.y * inv) * g.y, (v.z * inv) * g.z, (v.w * inv) * g.w);
    }
  }
  __syncthreads();
  unsigned long long best[MB];
#pragma unroll
  for (int b = 0; b < MB; ++b) best[b] = 0ull;
  const int rbeg = blockIdx.x * A.rows_per_cta, rend = min(A.V, rbeg + A.rows_per_cta);
  for (int r0 = rbeg + wid * RPW; r0 < rend; r0 += nw * RPW) {
    const float4* w4[RPW];
#pragma unroll
    for (int q = 0; q < RPW; ++q) w4[q] = reinterpret_cast<const float4*>(A.W + (size_t)min(r0 + q, rend - 1) * d);
    float acc[RPW][MB];
#pragma unroll
    for (int q = 0; q < RPW; ++q)
#pragma unroll
      for (int b = 0; b < MB; ++b) acc[q][b] = 0.f;
    for (int j0 = lane; j0 < K4; j0 += 32 * U) {
      float4 u[U][RPW];
#pragma unroll
      for (int t = 0; t < U; ++t)
#pragma unroll
        for (int q = 0; q < RPW; ++q)
          u[t][q] = (j0 + 32 * t < K4) ? __ldcs(w4[q] + j0 + 32 * t) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int t = 0; t < U; ++t) {
        if (j0 + 32 * t < K4) {
#pragma unroll
          for (int b = 0; b < MB; ++b) {
            if (b < A.B) {
              const float4 xv = reinterpret_cast<const float4*>(lb_smem + (size_t)b * d)[j0 + 32 * t];
#pragma unroll
              for (int q = 0; q < RPW; ++q) {
                acc[q][b] = fmaf(u[t][q].x, xv.x, acc[q][b]);
                acc[q][b] = fmaf(u[t][q].y, xv.y, acc[q][b]);
                acc[q][b] = fmaf(u[t][q].z, xv.z, acc[q][b]);
                acc[q][b] = fmaf(u[t][q].w, xv.w, acc[q][b]);
              }
            }
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < RPW; ++q) {
      const int r = r0 + q;
      if (r >= rend) break;
      const float bb = A.bias ? __ldg(A.bias + r) : 0.f;
#pragma unroll
      for (int b = 0; b < MB; ++b) {
        if (b < A.B) {
          const float v = warp_sum(acc[q][b]) + bb;
          if (lane == 0) A.logits[(size_t)b * A.V + r] = v;
          const unsigned long long key = amax_key(v, (unsigned)r + A.row_offset);
          best[b] = key > best[b] ? key : best[b];
        }
      }
    }
  }
  if (lane == 0)
    for (int b = 0; b < MB; ++b) wbest[wid][b] = best[b];
  __syncthreads();
  if (tid < A.B) {
    unsigned long long k = 0;
    for (int w = 0; w < nw; ++w) k = wbest[w][tid] > k ? wbest[w][tid] : k;
    A.part[(size_t)blockIdx.x * A.B + tid] = k;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = (atomicAdd(A.cnt, 1u) == gridDim.x - 1u);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int b = wid; b < A.B; b += nw) {
    unsigned long long k = 0;
    for (int c = lane; c < (int)gridDim.x; c += 32) {
      const unsigned long long v = __ldcg(A.part + (size_t)c * A.B + b);
      k = v > k ? v : k;
    }
    k = warp_max_u64(k);
    if (lane == 0) {
      if (A.argmax) A.argmax[b] = amax_index(k);
      if (A.keys) A.keys[b] = k;
    }
  }
  if (tid == 0) *A.cnt = 0u;  // ready for the next launch
}

// First-max argmax of each row of logits [B][V] (llm/forward.rs:262-271): one
// CTA of 512 threads per row (the tensor-core lm_head path).  Column i is
// vocab row i + row_offset; keys (nullable) receives each row's winning key.
__global__ void __launch_bounds__(512) k_argmax_rows(const float* logits, int V, unsigned* out,
                                                     unsigned row_offset, unsigned long long* keys) {
  __shared__ unsigned long long wb[16];
  pdl_wait();
  pdl_trigger();
  const float* row = logits + (size_t)blockIdx.x * V;
  unsigned long long best = 0ull;
#pragma unroll 4
  for (int i = threadIdx.x; i < V; i += 512) {
    const unsigned long long k = amax_key(__ldcg(row + i), (unsigned)i + row_offset);
    best = k > best ? k : best;
  }
  best = warp_max_u64(best);
  if ((threadIdx.x & 31) == 0) wb[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < 16; ++w) b = wb[w] > b ? wb[w] : b;
    if (out) out[blockIdx.x] = amax_index(b);
    if (keys) keys[blockIdx.x] = b;
  }
}

// The vocab-sharded argmax merge: keys_all[r][j] is rank r's best key (over
// its vocab rows) for gathered vector j; this rank's vector b is gathered
// vector rank*B + b.  The largest key over the ranks is the first maximum
// over the whole vocabulary (amax_key orders by value, then by lower index).
__global__ void k_shard_argmax(const unsigned long long* keys_all, int nranks, int B, int rank, unsigned* out) {
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    unsigned long long k = 0ull;
    for (int r = 0; r < nranks; ++r) {
      const unsigned long long v = keys_all[(size_t)r * nranks * B + (size_t)rank * B + b];
      k = v > k ? v : k;
    }
    out[b] = amax_index(k);
  }
}

}  // namespace gaje
