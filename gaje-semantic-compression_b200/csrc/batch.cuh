// batch.cuh -- one decode step for B independent streams of the same model
// (gaje_cuda_forward_batch: decode of a few streams after long prompts, and
// the per-rank body of multi-GPU serving).  Each stream has its own KV cache and position; the weights
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

#include <cuda_bf16.h>

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

// Batched decode attention, streamed: one CTA per (KV head, split, stream)
// over positions [t0, t0 + n) of the stream's cache (the step's own row
// included: the QKV kernel wrote it before this one).  The split's K rows and
// then its V rows pass through a ring of kAbStages shared-memory tiles of
// kAbTile rows (1-D TMA bulk copies, one mbarrier per stage), so loads run
// ahead of the arithmetic.  Scores: warp w takes positions 4w..4w+3 of a
// tile, lane l holds dims [VEC*l, VEC*l + VEC) of each of the G query heads in
// registers, and one butterfly reduce-scatter per warp turns the 4*G partial
// dots into one sum per lane.  Softmax over the split as in
// attention.rs:88-127 (split max, exp, sum).  P*V: warp j < G owns query head
// j, lane l its VEC dims, summing over the split's positions in order.  One
// split: out = O * (1/(l + 1e-12)); several: partials, and the last CTA of the
// (stream, KV head) combines them (attn_combine).
constexpr int kAbThreads = 256;
constexpr int kAbWarps = kAbThreads / 32;
constexpr int kAbTile = 32;       // positions per tile
constexpr int kAbStages = 4;
constexpr int kAbMaxChunk = 512;  // positions per split (scores held in shared memory)
constexpr int kAbMaxGroup = 8;    // query heads per KV head
__host__ __device__ inline size_t attn_batch2_smem(int G, int hd) {
  return 128 + size_t(kAbStages) * kAbTile * hd * 4 + size_t(G) * kAbMaxChunk * 4;
}
// Splits of a stream at context ctx when a launch allows at most ms.
__host__ __device__ inline void attn_batch2_splits(int ctx, int ms, int& nsplit, int& chunk) {
  int n0 = (ctx + 63) / 64;
  if (n0 > ms) n0 = ms;
  if (n0 < 1) n0 = 1;
  chunk = (ctx + n0 - 1) / n0;
  nsplit = (ctx + chunk - 1) / chunk;
}

// The combine of the last CTA of (stream, KV head): weights e^{m_s - M},
// out = (sum_s O_s w_s) * (1/(sum_s l_s w_s + 1e-12)).
__device__ __forceinline__ void attn_combine(const float* part_o, const float* part_ml, int G, int hd, int nsplit,
                                             float* out, float* wsh, float* linv) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int idx = threadIdx.x; idx < G * nsplit; idx += blockDim.x) {
    const int j = idx / nsplit, r = idx - j * nsplit;
    wsh[idx] = __ldcg(part_ml + ((size_t)r * G + j) * 2);
  }
  __syncthreads();
  for (int j = wid; j < G; j += nw) {
    float M = -INFINITY;
    for (int r = lane; r < nsplit; r += kWarp) M = fmaxf(M, wsh[j * nsplit + r]);
    M = warp_max(M);
    float Lsum = 0.f;
    for (int r = lane; r < nsplit; r += kWarp) {
      const float w = expf(wsh[j * nsplit + r] - M);
      wsh[j * nsplit + r] = w;
      Lsum += __ldcg(part_ml + ((size_t)r * G + j) * 2 + 1) * w;
    }
    Lsum = warp_sum(Lsum);
    if (lane == 0) linv[j] = 1.0f / (Lsum + 1e-12f);
  }
  __syncthreads();
  // up to four outputs per thread at once, eight partials each: 32 loads in
  // flight; every output adds its splits in the same order as one at a time
  const int total = G * hd, nt = blockDim.x;
  for (int base = threadIdx.x; base < total; base += 4 * nt) {
    float O0[4] = {0.f, 0.f, 0.f, 0.f}, O1[4] = {0.f, 0.f, 0.f, 0.f};
    for (int r0 = 0; r0 < nsplit; r0 += 8) {
      float v[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int idx = base + u * nt;  // = j * hd + e: split r at part_o + r*G*hd + idx
#pragma unroll
        for (int k = 0; k < 8; ++k)
          v[u][k] = (idx < total && r0 + k < nsplit) ? __ldcg(part_o + (size_t)(r0 + k) * total + idx) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int idx = base + u * nt;
        if (idx >= total) continue;
        const int j = idx / hd;
#pragma unroll
        for (int k = 0; k < 8; k += 2) {
          if (r0 + k < nsplit) O0[u] += v[u][k] * wsh[j * nsplit + r0 + k];
          if (r0 + k + 1 < nsplit) O1[u] += v[u][k + 1] * wsh[j * nsplit + r0 + k + 1];
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int idx = base + u * nt;
      if (idx < total) out[idx] = (O0[u] + O1[u]) * linv[idx / hd];
    }
  }
}

template <int VEC>
__global__ void __launch_bounds__(kAbThreads, 2) k_attn_batch2(AttnBatchArgs B) {
  constexpr int HD = 32 * VEC;
  extern __shared__ __align__(128) unsigned char ab_smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(ab_smem);  // [kAbStages]
  float* tiles = reinterpret_cast<float*>(ab_smem + 128);   // [kAbStages][kAbTile][HD]
  float* ps = tiles + (size_t)kAbStages * kAbTile * HD;     // [G][kAbMaxChunk]
  __shared__ float ml_s[2 * kAbMaxGroup];
  __shared__ float wsh[kAbMaxGroup * kAttnMaxSplits];
  __shared__ float linv[kAbMaxGroup];
  __shared__ int is_last;
  const int g = blockIdx.x, s = blockIdx.y, b = blockIdx.z;
  const int nkv = B.cache.nkv, G = B.nh / nkv;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  pdl_wait();
  pdl_trigger();
  const int ctx = int(B.bs.pos[b]) + 1;
  int nsplit, chunk;
  attn_batch2_splits(ctx, B.max_splits, nsplit, chunk);
  if (s >= nsplit) return;
  const int t0 = s * chunk, n = min(ctx, t0 + chunk) - t0;
  const int ntile = (n + kAbTile - 1) / kAbTile;
  const int nitems = 2 * ntile;  // K tiles, then V tiles
  const unsigned sid = B.bs.sid[b];
  const float* kbase = B.cache.k + B.cache.row(sid, B.layer, g, unsigned(t0));
  const float* vbase = B.cache.v + B.cache.row(sid, B.layer, g, unsigned(t0));
  if (tid == 0) {
    for (int i = 0; i < kAbStages; ++i) mbar_init(full + i, 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int it) {  // thread 0: item it into stage it % kAbStages
    const int k = it < ntile ? it : it - ntile;
    const int rows = min(kAbTile, n - k * kAbTile);
    const float* src = (it < ntile ? kbase : vbase) + (size_t)k * kAbTile * HD;
    const uint32_t bytes = uint32_t(rows) * HD * 4;
    uint64_t* bar = full + (it % kAbStages);
    mbar_expect_tx(bar, bytes);
    // cache rows are read once per step: evict-first keeps L2 for the reused data
    bulk_g2s_hint(tiles + (size_t)(it % kAbStages) * kAbTile * HD, src, bytes, bar, l2_policy_evict_first());
  };
  if (tid == 0)
    for (int it = 0; it < min(kAbStages, nitems); ++it) issue(it);
  // this lane's dims of the G query heads
  float q[kAbMaxGroup][VEC];
  const float* qg = B.q + (size_t)b * B.nh * HD + (size_t)g * G * HD;
#pragma unroll
  for (int j = 0; j < kAbMaxGroup; ++j)
#pragma unroll
    for (int v = 0; v < VEC; ++v) q[j][v] = j < G ? __ldcg(qg + (size_t)j * HD + VEC * lane + v) : 0.f;
  bool ok = true;
  // ---- scores: warp w, positions 4w..4w+3 of each tile
  for (int k = 0; k < ntile; ++k) {
    if (!mbar_wait(full + (k % kAbStages), (k / kAbStages) & 1)) ok = false;
    const float* tk = tiles + (size_t)(k % kAbStages) * kAbTile * HD;
    float part[4 * kAbMaxGroup];  // value (head j, position 4w+tq) at [j*4 + tq]
#pragma unroll
    for (int tq = 0; tq < 4; ++tq) {
      const int t = 4 * wid + tq;
      float kv[VEC];
      if constexpr (VEC == 4) {
        const float4 x = reinterpret_cast<const float4*>(tk + (size_t)t * HD)[lane];
        kv[0] = x.x; kv[1] = x.y; kv[2] = x.z; kv[3] = x.w;
      } else if constexpr (VEC == 2) {
        const float2 x = reinterpret_cast<const float2*>(tk + (size_t)t * HD)[lane];
        kv[0] = x.x; kv[1] = x.y;
      } else {
        kv[0] = tk[(size_t)t * HD + lane];
      }
#pragma unroll
      for (int j = 0; j < kAbMaxGroup; ++j) {
        float a = 0.f;
#pragma unroll
        for (int v = 0; v < VEC; ++v) a = fmaf(q[j][v], kv[v], a);
        part[j * 4 + tq] = a;
      }
    }
    // butterfly reduce-scatter of 32 values over 32 lanes: lane l ends with
    // the full sum of value l
#pragma unroll
    for (int o = 16, h = 16; o >= 1; o >>= 1, h >>= 1) {
      const bool up = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < h; ++i) {
        const float send = up ? part[i] : part[i + h];
        const float keep = up ? part[i + h] : part[i];
        part[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
    {
      // level o keeps the half of the values selected by lane bit o, so after
      // the five levels lane l holds value index l
      const int j = lane >> 2, tq = lane & 3;
      const int t = k * kAbTile + 4 * wid + tq;
      if (j < G && t < n) ps[j * kAbMaxChunk + t] = part[0] * B.scale;
    }
    __syncthreads();  // the stage is consumed
    if (tid == 0 && k + kAbStages < nitems) issue(k + kAbStages);
  }
  // ---- softmax over the split: warp j < G owns head j
  if (wid < G) {
    float* pr = ps + wid * kAbMaxChunk;
    float m = -INFINITY;
    for (int t = lane; t < n; t += kWarp) m = fmaxf(m, pr[t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < n; t += kWarp) {
      const float e = expf(pr[t] - m);
      pr[t] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      ml_s[2 * wid] = m;
      ml_s[2 * wid + 1] = l;
    }
  }
  __syncthreads();
  // ---- P*V
  float acc[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) acc[v] = 0.f;
  for (int k = 0; k < ntile; ++k) {
    const int it = ntile + k;
    if (!mbar_wait(full + (it % kAbStages), (it / kAbStages) & 1)) ok = false;
    const float* tv = tiles + (size_t)(it % kAbStages) * kAbTile * HD;
    if (wid < G) {
      const float* pr = ps + wid * kAbMaxChunk + k * kAbTile;
      const int rows = min(kAbTile, n - k * kAbTile);
      for (int t = 0; t < rows; ++t) {
        const float p = pr[t];
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[v] = fmaf(p, tv[(size_t)t * HD + VEC * lane + v], acc[v]);
      }
    }
    __syncthreads();
    if (tid == 0 && it + kAbStages < nitems) issue(it + kAbStages);
  }
  if (!ok) return;  // a copy that never landed: the step's outputs stay stale (bounded waits, no hang)
  float* outg = B.out + (size_t)b * B.nh * HD + (size_t)g * G * HD;
  if (nsplit == 1) {
    if (wid < G) {
      const float inv = 1.0f / (ml_s[2 * wid + 1] + 1e-12f);
#pragma unroll
      for (int v = 0; v < VEC; ++v) outg[(size_t)wid * HD + VEC * lane + v] = acc[v] * inv;
    }
    return;
  }
  const size_t pbase = ((size_t)b * nkv + g) * kAttnMaxSplits;  // (stream, KV head) partials
  float* po = B.part_o + (pbase + s) * G * HD;
  float* pml = B.part_ml + (pbase + s) * G * 2;
  if (wid < G) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) po[(size_t)wid * HD + VEC * lane + v] = acc[v];
    if (lane == 0) {
      pml[2 * wid] = ml_s[2 * wid];
      pml[2 * wid + 1] = ml_s[2 * wid + 1];
    }
  }
  __threadfence();
  __syncthreads();
  unsigned* cnt = B.cnt + (size_t)b * nkv + g;
  if (tid == 0) is_last = (atomicAdd(cnt, 1u) == (unsigned)nsplit - 1u);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  attn_combine(B.part_o + pbase * G * HD, B.part_ml + pbase * G * 2, G, HD, nsplit, outg, wsh, linv);
  if (tid == 0) *cnt = 0u;  // ready for the next launch
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

// The same causal prefill attention on the tensor cores (legacy mma.sync
// m16n8k16 bf16, f32 accumulate), for head_dim 64 and 128.  A warp owns 16
// (row, query head) pairs of the CTA's 96 -- the pairing of k_attn_prefill
// -- with its q rows as bf16 hi/lo A fragments in registers; K/V arrive in
// 64-position tiles (cp.async brings the next tile's f32 rows into a staging
// buffer while the current tile's MMAs run), split into bf16 hi/lo planes in
// padded shared memory and read with ldmatrix (transposed for V).  Scores S = q.k take three MMAs
// per 16-wide k-step (hi.hi + hi.lo + lo.hi, the products' dropped terms
// below 2^-16 relative), then scale, the causal mask and the running
// max/sum in f32 registers; the probabilities, split hi/lo the same way,
// are fed straight from the score accumulators as the A fragments of P.V
// (three MMAs again).  The register-resident P is why this uses mma.sync
// rather than tcgen05 (whose A operand would have to round-trip through
// shared or tensor memory for every 64-position tile).
constexpr int kAtWarps = kApQG / 16;        // 6 warps x 16 pairs
constexpr int kAtThreads = kAtWarps * 32;
constexpr int kAtT = 64;                    // key positions per tile
__host__ __device__ constexpr int attn_tc_stride(int hd) { return hd + 8; }  // bf16 per smem row (ldmatrix conflict-free)
// bf16 hi/lo K and V planes + the f32 staging of the next tile's K and V rows
__host__ __device__ constexpr size_t attn_tc_smem(int hd) {
  return size_t(4) * kAtT * attn_tc_stride(hd) * 2 + size_t(2) * kAtT * hd * 4;
}

__device__ __forceinline__ void at_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void at_ldsm4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void at_ldsm4t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// (x, y) -> bf16x2 hi (x in the low half) and the residues' bf16x2 lo.
__device__ __forceinline__ void at_split2(float x, float y, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
  const float2 f = __bfloat1622float2(h);
  const __nv_bfloat162 l = __floats2bfloat162_rn(x - f.x, y - f.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

template <int HD>
__global__ void __launch_bounds__(kAtThreads, 1) k_attn_prefill_tc(AttnPrefillArgs A) {
  static_assert(HD == 64 || HD == 128, "head_dim");
  constexpr int SR = attn_tc_stride(HD), KS = HD / 16, ND = HD / 8;
  extern __shared__ __align__(16) unsigned char at_smem[];
  __nv_bfloat16* Khi = reinterpret_cast<__nv_bfloat16*>(at_smem);
  __nv_bfloat16* Klo = Khi + kAtT * SR;
  __nv_bfloat16* Vhi = Klo + kAtT * SR;
  __nv_bfloat16* Vlo = Vhi + kAtT * SR;
  float* Kst = reinterpret_cast<float*>(Vlo + kAtT * SR);  // [kAtT][HD] f32 staging
  float* Vst = Kst + kAtT * HD;
  const int G = A.nh / A.nkv, QB = attn_prefill_qb(G), QG = QB * G;
  const int gk = blockIdx.y, m0 = (gridDim.x - 1 - blockIdx.x) * QB;  // longest causal spans first
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  pdl_wait();
  pdl_trigger();
  const int last = min(A.n, m0 + QB) - 1;
  // this thread's two pairs (rows gq, gq + 8 of the warp's 16): the last position each sees
  int plim[2];
  const float* qrow[2];
  float* orow[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int qh = 16 * wid + gq + 8 * h, i = qh / G, j = qh - i * G;
    const bool live = qh < QG && m0 + i <= last;
    plim[h] = live ? A.p0 + m0 + i : -1;
    const size_t off = live ? (size_t)(m0 + i) * A.nh * HD + (size_t)(gk * G + j) * HD : 0;
    qrow[h] = live ? A.q + off : nullptr;
    orow[h] = live ? A.out + off : nullptr;
  }
  int wlim = max(plim[0], plim[1]);
#pragma unroll
  for (int o = 16; o; o >>= 1) wlim = max(wlim, __shfl_xor_sync(0xffffffffu, wlim, o));
  // q A fragments: k-step kk, regs (row gq, dims 2tq..), (row gq+8, ..), (row gq, +8), (row gq+8, +8)
  uint32_t qa[KS][4], ql[KS][4];
#pragma unroll
  for (int kk = 0; kk < KS; ++kk)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int h = r & 1, dim = 16 * kk + 2 * tq + 8 * (r >> 1);
      float2 v = make_float2(0.f, 0.f);
      if (qrow[h]) v = __ldcg(reinterpret_cast<const float2*>(qrow[h] + dim));
      at_split2(v.x, v.y, qa[kk][r], ql[kk][r]);
    }
  float o[ND][4];
#pragma unroll
  for (int nd = 0; nd < ND; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const int maxpos = A.p0 + last;
  const float* kbase = A.kc + (size_t)gk * A.max_ctx * HD;
  const float* vbase = A.vc + (size_t)gk * A.max_ctx * HD;
  const uint32_t sKhi = smem_u32(Khi), sKlo = smem_u32(Klo), sVhi = smem_u32(Vhi), sVlo = smem_u32(Vlo);
  // ldmatrix row addresses of this lane: matrix mi = lane / 8, row ri = lane % 8
  const int mi = lane >> 3, ri = lane & 7;
  const uint32_t koff = uint32_t(((mi >> 1) * 8 + ri) * SR + (mi & 1) * 8) * 2u;  // + 16 pos per pair, + 16 dims per k-step
  const uint32_t voff = uint32_t(((mi & 1) * 8 + ri) * SR + (mi >> 1) * 8) * 2u;  // + 16 pos per k-step, + 16 dims per pair
  // a tile's rows (positions <= maxpos) into the staging buffer: this thread's 16-byte pieces
  auto stage = [&](int ts) {
    for (int idx = tid; idx < kAtT * (HD / 4); idx += kAtThreads) {
      const int jp = idx / (HD / 4), e4 = idx - jp * (HD / 4);
      if (ts + jp <= maxpos) {
        cp_async16(Kst + 4 * idx, kbase + (size_t)(ts + jp) * HD + 4 * e4);
        cp_async16(Vst + 4 * idx, vbase + (size_t)(ts + jp) * HD + 4 * e4);
      }
    }
  };
  stage(0);
  for (int t0 = 0; t0 <= maxpos; t0 += kAtT) {
    cp_async_wait_all();  // this thread's pieces of tile t0 have landed
    __syncthreads();      // ... everyone's, and the previous tile's planes are consumed
    for (int idx = tid; idx < kAtT * (HD / 4); idx += kAtThreads) {
      const int jp = idx / (HD / 4), e4 = idx - jp * (HD / 4);
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (t0 + jp <= maxpos) {
        kv = reinterpret_cast<const float4*>(Kst)[idx];
        vv = reinterpret_cast<const float4*>(Vst)[idx];
      }
      uint2 h2, l2;
      at_split2(kv.x, kv.y, h2.x, l2.x);
      at_split2(kv.z, kv.w, h2.y, l2.y);
      *reinterpret_cast<uint2*>(Khi + jp * SR + 4 * e4) = h2;
      *reinterpret_cast<uint2*>(Klo + jp * SR + 4 * e4) = l2;
      at_split2(vv.x, vv.y, h2.x, l2.x);
      at_split2(vv.z, vv.w, h2.y, l2.y);
      *reinterpret_cast<uint2*>(Vhi + jp * SR + 4 * e4) = h2;
      *reinterpret_cast<uint2*>(Vlo + jp * SR + 4 * e4) = l2;
    }
    __syncthreads();  // planes ready, staging free
    if (t0 + kAtT <= maxpos) stage(t0 + kAtT);  // the next tile's rows land during this tile's MMAs
    if (t0 > wlim) continue;  // no pair of this warp sees the tile (warp-uniform)
    // S = q k^T over the tile: n-tiles nt of 8 positions
    float sc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk)
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const uint32_t a = koff + uint32_t(16 * np * SR + 16 * kk) * 2u;
        uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
        at_ldsm4(sKhi + a, h0, h1, h2, h3);
        at_ldsm4(sKlo + a, l0, l1, l2, l3);
        at_mma(sc[2 * np], qa[kk], h0, h1);
        at_mma(sc[2 * np], qa[kk], l0, l1);
        at_mma(sc[2 * np], ql[kk], h0, h1);
        at_mma(sc[2 * np + 1], qa[kk], h2, h3);
        at_mma(sc[2 * np + 1], qa[kk], l2, l3);
        at_mma(sc[2 * np + 1], ql[kk], h2, h3);
      }
    // scale, causal mask, running max / sum (rows gq, gq + 8: a quad of lanes per row)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int pos = t0 + nt * 8 + 2 * tq + e;
          const float v = pos <= plim[h] ? sc[nt][2 * h + e] * A.scale : -INFINITY;
          sc[nt][2 * h + e] = v;
          mx = fmaxf(mx, v);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(mrow[h], mx);
      float alpha = 1.f, psum = 0.f;
      if (mn > -INFINITY) {  // pads and rows that see nothing yet keep p = 0
        alpha = expf(mrow[h] - mn);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float p = expf(sc[nt][2 * h + e] - mn);
            sc[nt][2 * h + e] = p;
            psum += p;
          }
      } else {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) sc[nt][2 * h] = sc[nt][2 * h + 1] = 0.f;
      }
      psum += __shfl_xor_sync(0xffffffffu, psum, 1);
      psum += __shfl_xor_sync(0xffffffffu, psum, 2);
      lrow[h] = lrow[h] * alpha + psum;
      mrow[h] = mn;
#pragma unroll
      for (int nd = 0; nd < ND; ++nd) {
        o[nd][2 * h] *= alpha;
        o[nd][2 * h + 1] *= alpha;
      }
    }
    // O += P V: k-steps of 16 positions, P's A fragments straight from the score accumulators
#pragma unroll
    for (int kp = 0; kp < 4; ++kp) {
      uint32_t pa[4], pl[4];
      at_split2(sc[2 * kp][0], sc[2 * kp][1], pa[0], pl[0]);
      at_split2(sc[2 * kp][2], sc[2 * kp][3], pa[1], pl[1]);
      at_split2(sc[2 * kp + 1][0], sc[2 * kp + 1][1], pa[2], pl[2]);
      at_split2(sc[2 * kp + 1][2], sc[2 * kp + 1][3], pa[3], pl[3]);
#pragma unroll
      for (int dp = 0; dp < ND / 2; ++dp) {
        const uint32_t a = voff + uint32_t(16 * kp * SR + 16 * dp) * 2u;
        uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
        at_ldsm4t(sVhi + a, h0, h1, h2, h3);
        at_ldsm4t(sVlo + a, l0, l1, l2, l3);
        at_mma(o[2 * dp], pa, h0, h1);
        at_mma(o[2 * dp], pa, l0, l1);
        at_mma(o[2 * dp], pl, h0, h1);
        at_mma(o[2 * dp + 1], pa, h2, h3);
        at_mma(o[2 * dp + 1], pa, l2, l3);
        at_mma(o[2 * dp + 1], pl, h2, h3);
      }
    }
  }
  // out = O / (sum + 1e-12) (attention.rs:106-127)
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (!orow[h]) continue;
    const float inv = 1.0f / (lrow[h] + 1e-12f);
#pragma unroll
    for (int nd = 0; nd < ND; ++nd)
      *reinterpret_cast<float2*>(orow[h] + nd * 8 + 2 * tq) = make_float2(o[nd][2 * h] * inv, o[nd][2 * h + 1] * inv);
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
  int flush;            // 1: flush |t| < 1e-6 to 0 before the bias (a Q8_0 lm_head)
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
          float v = warp_sum(acc[q][b]);
          if (A.flush) v = flush_small(v);
          v += bb;
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
