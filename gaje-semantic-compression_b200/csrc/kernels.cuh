// kernels.cuh -- sm_100a kernels of the batch-1 decode step.
//
// One decode step of GenomicLLM::forward_core (src/nn/llm/forward.rs:7-63) is
// five kernels per block plus the lm_head:
//   k_qkv     RMSNorm prologue (norm.rs:17-87) + Q4_0 GEMV of attn_qkv
//             (genomic.rs:267-336, flush + bias of linear/forward.rs:84-115)
//             + RoPE (attention.rs:62-84) + KV-cache append (attention.rs:85-86)
//   k_attn    split-K flash-decode GQA attention (attention.rs:88-127); the
//             last CTA of each KV head combines the splits
//   k_oproj   Q4_0 GEMV of attn_output + residual add (block/forward.rs:76-82)
//   k_gateup  RMSNorm prologue + Q4_0 GEMV of ffn_gate_up, gate row n and up
//             row ff+n in one warp, SwiGLU epilogue (activation.rs:35-51)
//   k_down    Q4_0 GEMV of ffn_down + residual add (block/forward.rs:124-136)
//   k_lmhead  final RMSNorm + FP32 GEMV (dot.rs:46-67) + first-max argmax
//             (llm/forward.rs:262-271); the last CTA finishes the argmax
// Optional: k_kwta (lut.rs:45-61) on the logits or on the hidden state.
//
// Numerics: the file is compiled with --fmad=false, so every FMA below is an
// explicit fmaf(); products and sums elsewhere round exactly as written, as
// in the Rust reference (which never contracts).  The Q4_0 dequantised weight
// is fmaf(q, scale, min) -- bit-identical to the AVX2 kernel's fused dequant
// (genomic.rs:298).  Summation order differs from the AVX2 8-lane order, so
// dot products agree to rounding, not bit for bit.
//
// Device errors are status words, never traps: NaN guards (block/forward.rs
// :11-140) record the earliest (layer, check) with atomicMin.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gaje {

constexpr int kWarp = 32;
constexpr int kGemvThreads = 256;       // 8 warps per GEMV CTA
constexpr int kAttnThreads = 128;
constexpr int kAttnMinChunk = 16;       // positions per attention split (minimum)
constexpr int kAttnMaxSplits = 64;
constexpr int kAttnMaxGroup = 16;       // q heads per kv head
constexpr int kLmThreads = 256;
constexpr int kKwtaThreads = 1024;

// NaN guard codes, in the order block/forward.rs checks them.
enum NanCheck : unsigned {
  kNanInput = 0,      // "Input x is NaN"                    (:11-13)
  kNanAttnNorm = 1,   // "NaN after attn rms_norm"           (:22-24)
  kNanUp = 2,         // "NaN in up"                         (:97-99)
  kNanFfnOut = 3,     // "NaN in ffn_out"                    (:111-113)
  kNanProjFfn = 4,    // "NaN in projected_ffn"              (:128-130)
  kNanResidual = 5,   // "NaN after projected_ffn addition"  (:138-140)
};

// Per-model device state: the only values a replayed step graph reads from or
// writes to besides activations and the KV cache.
struct DevState {
  unsigned pos;        // cache length before this step (= position of the new token)
  unsigned token;      // input token id of this step
  unsigned argmax;     // first index of the max logit of the last step
  unsigned nan_code;   // 0xFFFFFFFF, or pos*4096 + layer*8 + check of the first NaN guard
  unsigned hist_len;   // entries written to the token history
  unsigned pad[3];
};

// A Q4_0 matrix in the engine's layout: per row, nb = K/32 blocks; qs[row][b]
// holds the block's 16 nibble bytes unchanged (element 2k = low nibble of
// byte k), sm[row][b] = f16 scale | f16 min << 16.  Same 20 bytes per block as
// the file, split into 16-byte-aligned arrays so a lane reads a block with one
// 128-bit load.
struct Q4View {
  const uint4* qs;
  const uint32_t* sm;
  const float* bias;  // [N] or nullptr
  int N, K, nb;
};

struct LayerW {
  Q4View qkv, wo, gate_up, down;
  const float* attn_norm;
  const float* ffn_norm;
  float* kc;  // [nkv][max_ctx][hd]
  float* vc;
};

struct StepParams {
  int d, nh, nkv, hd, ff, V, max_ctx, n_layers;
  float eps, attn_scale;
  int rope_split, use_genomic_norm;
  const float* embd;     // f32 [V][d]
  const float* lm_head;  // f32 [V][d]
  const float* lm_bias;  // [V] or nullptr
  const float* out_norm;
  const float2* rope;    // [max_ctx][hd/2] (cos, sin) from host libm
  float* x;              // residual stream [d]
  float* q;              // rotated q [nh*hd]
  float* attn;           // attention output [nh*hd]
  float* act;            // SwiGLU output [ff]
  float* logits;         // [V]
  float* part_o;         // [nkv][kAttnMaxSplits][G][hd]
  float* part_ml;        // [nkv][kAttnMaxSplits][G][2]
  unsigned* attn_cnt;    // [nkv]
  unsigned long long* amax_part;  // [lm grid]
  unsigned* amax_cnt;
  unsigned* tok_hist;    // [hist_cap]
  unsigned hist_cap;
  DevState* st;
};

// ------------------------------------------------------------------ helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  return v;
}

// Block-wide sum for blockDim.x <= 1024; `red` holds 32 floats of smem.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.0f;
  return warp_sum(t);
}

// Rust f32::clamp: NaN passes through.
__device__ __forceinline__ float rclamp(float v, float lo, float hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}

// The reference's |sum| < 1e-6 -> 0 flush of every Q4_0/Q8_0 row dot
// (genomic.rs:331-335); NaN is kept.
__device__ __forceinline__ float flush_small(float v) { return fabsf(v) < 1e-6f ? 0.0f : v; }

// XOR swizzle of an activation vector in shared memory: the eight float4
// chunks of each 32-element block are permuted by the block index so that the
// eight lanes of a quarter warp, each reading chunk c of a different block,
// hit eight different bank groups.
__device__ __forceinline__ int swz(int i) {
  const int b = i >> 5;
  return (i & ~31) | ((((i >> 2) & 7) ^ (b & 7)) << 2) | (i & 3);
}

// Exact float of a 4-bit code: 2^23 + q has q in its low mantissa bits.
__device__ __forceinline__ float nib(uint32_t w, int shift) {
  return __uint_as_float(((w >> shift) & 0xFu) | 0x4B000000u) - 8388608.0f;
}

__device__ __forceinline__ void unpack_sm(uint32_t smv, float& scale, float& mn) {
  scale = __half2float(__ushort_as_half((unsigned short)(smv & 0xFFFFu)));
  mn = __half2float(__ushort_as_half((unsigned short)(smv >> 16)));
}

// One lane's share of a row dot: all 32 weights of block b against the
// swizzled activations xs.  Element 8w+4h+j of the block is nibble j of the
// 16-bit half h of word w (low nibble of byte k is element 2k).
__device__ __forceinline__ float q4_block_dot(const uint4 q, uint32_t smv, const float* xs, int b) {
  float scale, mn;
  unpack_sm(smv, scale, mn);
  const float4* x4 = reinterpret_cast<const float4*>(xs + (b << 5));
  const int sw = b & 7;
  const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const float4 xv = x4[c ^ sw];
    const uint32_t w = wd[c >> 1];
    const int s = (c & 1) << 4;
    a0 = fmaf(fmaf(nib(w, s + 0), scale, mn), xv.x, a0);
    a1 = fmaf(fmaf(nib(w, s + 4), scale, mn), xv.y, a1);
    a2 = fmaf(fmaf(nib(w, s + 8), scale, mn), xv.z, a2);
    a3 = fmaf(fmaf(nib(w, s + 12), scale, mn), xv.w, a3);
  }
  return (a0 + a1) + (a2 + a3);
}

// Full row dot of one Q4_0 row by one warp (lanes stride the blocks).  The
// returned value is flushed and biased like compute_single_row.
__device__ __forceinline__ float q4_row(const Q4View& W, int row, const float* xs, int lane) {
  const uint4* qs = W.qs + (size_t)row * W.nb;
  const uint32_t* sm = W.sm + (size_t)row * W.nb;
  float acc = 0.f;
#pragma unroll 4
  for (int b = lane; b < W.nb; b += kWarp) acc += q4_block_dot(__ldg(qs + b), __ldg(sm + b), xs, b);
  float y = flush_small(warp_sum(acc));
  if (W.bias) y += __ldg(W.bias + row);
  return y;
}

// Two rows at once (more loads in flight per lane).
__device__ __forceinline__ void q4_row2(const Q4View& W, int r0, int r1, const float* xs, int lane,
                                        float& y0, float& y1) {
  const uint4* qs0 = W.qs + (size_t)r0 * W.nb;
  const uint4* qs1 = W.qs + (size_t)r1 * W.nb;
  const uint32_t* sm0 = W.sm + (size_t)r0 * W.nb;
  const uint32_t* sm1 = W.sm + (size_t)r1 * W.nb;
  float a = 0.f, c = 0.f;
#pragma unroll 2
  for (int b = lane; b < W.nb; b += kWarp) {
    const uint4 qa = __ldg(qs0 + b), qc = __ldg(qs1 + b);
    const uint32_t sa = __ldg(sm0 + b), sc = __ldg(sm1 + b);
    a += q4_block_dot(qa, sa, xs, b);
    c += q4_block_dot(qc, sc, xs, b);
  }
  y0 = flush_small(warp_sum(a));
  y1 = flush_small(warp_sum(c));
  if (W.bias) {
    y0 += __ldg(W.bias + r0);
    y1 += __ldg(W.bias + r1);
  }
}

// NaN guard code: position * 4096 + layer * 8 + check, so atomicMin keeps the
// first failing check of the first failing step, the one the reference stops at.
__device__ __forceinline__ void nan_flag(DevState* st, int layer, unsigned check) {
  atomicMin(&st->nan_code, st->pos * 4096u + unsigned(layer) * 8u + check);
}

// RMSNorm of src[0..n) into swizzled smem xs (norm.rs:17-87):
// inv = 1/sqrt(sum(x^2)/n + eps); out = (x*inv)*w.  The sum is a tree here
// (the reference uses an 8-lane FMA sweep), so inv agrees to rounding.
// Returns true if src held a NaN (nan_in) or the output did (nan_out).
__device__ __forceinline__ void rmsnorm_smem(const float* __restrict__ src, const float* __restrict__ w,
                                             float eps, int n, float* xs, float* red, bool& nan_in,
                                             bool& nan_out) {
  float ss = 0.f;
  int bad = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = src[i];
    ss = fmaf(v, v, ss);
    bad |= (v != v);
  }
  ss = block_sum(ss, red);
  const int any_bad_in = __syncthreads_or(bad);
  const float inv = 1.0f / sqrtf(ss / (float)n + eps);
  int bad_out = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float o = (src[i] * inv) * w[i];
    bad_out |= (o != o);
    xs[swz(i)] = o;
  }
  nan_out = __syncthreads_or(bad_out) != 0;
  nan_in = any_bad_in != 0;
}

// ------------------------------------------------------------------ kernels

// attn_qkv with the attn_norm prologue; layer 0 reads the embedding row of
// the step's token (get_row_core, linear/forward.rs:195-209: row token % V)
// and also materialises the residual stream x.
__global__ void __launch_bounds__(kGemvThreads) k_qkv(StepParams P, LayerW W, int layer) {
  extern __shared__ float smem[];
  float* xs = smem;           // [d] swizzled
  __shared__ float red[32];
  const unsigned pos = P.st->pos;
  const float* src = P.x;
  if (layer == 0) {
    const unsigned tok = P.st->token % (unsigned)P.V;
    src = P.embd + (size_t)tok * P.d;
    if (blockIdx.x == 0)
      for (int i = threadIdx.x; i < P.d; i += blockDim.x) P.x[i] = src[i];
  }
  bool nan_in, nan_out;
  rmsnorm_smem(src, W.attn_norm, P.eps, P.d, xs, red, nan_in, nan_out);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (nan_in) nan_flag(P.st, layer, kNanInput);
    if (nan_out) nan_flag(P.st, layer, kNanAttnNorm);
  }
  const int lane = threadIdx.x & 31;
  const int half = P.hd >> 1;
  const int npairs = W.qkv.N >> 1;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const float2* rope = P.rope + (size_t)pos * half;
  for (int p = gw; p < npairs; p += nwarps) {
    const int head = p / half, i = p - head * half;  // head over q, k, v heads
    const int r0 = head * P.hd + (P.rope_split ? i : 2 * i);
    const int r1 = r0 + (P.rope_split ? half : 1);
    float y0, y1;
    q4_row2(W.qkv, r0, r1, xs, lane, y0, y1);
    if (lane == 0) {
      if (head < P.nh + P.nkv) {  // RoPE on q and k: v0*cos - v1*sin, v0*sin + v1*cos
        const float2 cs = rope[i];
        const float o0 = y0 * cs.x - y1 * cs.y;
        const float o1 = y0 * cs.y + y1 * cs.x;
        y0 = o0;
        y1 = o1;
      }
      const int c0 = r0 - head * P.hd, c1 = r1 - head * P.hd;
      if (head < P.nh) {
        P.q[r0] = y0;
        P.q[r1] = y1;
      } else {
        const bool is_k = head < P.nh + P.nkv;
        const int g = is_k ? head - P.nh : head - P.nh - P.nkv;
        float* c = (is_k ? W.kc : W.vc) + ((size_t)g * P.max_ctx + pos) * P.hd;
        c[c0] = y0;
        c[c1] = y1;
      }
    }
  }
}

// Split bookkeeping shared by the attention kernel and its host wrapper.
__host__ __device__ __forceinline__ void attn_splits(int ctx, int& nsplit, int& chunk) {
  int n0 = (ctx + kAttnMinChunk - 1) / kAttnMinChunk;
  if (n0 > kAttnMaxSplits) n0 = kAttnMaxSplits;
  if (n0 < 1) n0 = 1;
  chunk = (ctx + n0 - 1) / n0;
  nsplit = (ctx + chunk - 1) / chunk;
}

// One CTA per (kv head g, split s).  Scores for the G query heads of the group
// over the split's positions, exp against the split max, unnormalised P*V;
// the last CTA of the group to finish combines the splits:
//   out = (sum_s O_s e^{m_s-M}) * (1/(sum_s l_s e^{m_s-M} + 1e-12))
// (the reference's inv_s = 1/(sum_e + 1e-12), attention.rs:110).
__device__ __forceinline__ void attn_core(const float* __restrict__ q, const float* __restrict__ kc,
                                          const float* __restrict__ vc, float* __restrict__ out,
                                          int ctx, int cache_stride, int nh, int nkv, int hd,
                                          float scale, float* part_o, float* part_ml,
                                          unsigned* cnt) {
  extern __shared__ float smem[];
  const int G = nh / nkv;
  const int g = blockIdx.x, s = blockIdx.y;
  int nsplit, chunk;
  attn_splits(ctx, nsplit, chunk);
  if (s >= nsplit) return;
  const int t0 = s * chunk;
  const int n = min(ctx, t0 + chunk) - t0;
  float* qs = smem;            // [G][hd]
  float* ps = qs + G * hd;     // [G][chunk]
  __shared__ float mls[2 * kAttnMaxGroup];
  __shared__ int is_last;
  for (int i = threadIdx.x; i < G * hd; i += blockDim.x) qs[i] = q[(size_t)g * G * hd + i];
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const float* kbase = kc + ((size_t)g * cache_stride + t0) * hd;
  const float* vbase = vc + ((size_t)g * cache_stride + t0) * hd;
  // scores: one warp per position, lanes across head_dim
  for (int t = wid; t < n; t += nw) {
    const float* kr = kbase + (size_t)t * hd;
    for (int j = 0; j < G; ++j) {
      float a = 0.f;
      for (int e = lane; e < hd; e += kWarp) a = fmaf(qs[j * hd + e], kr[e], a);
      a = warp_sum(a);
      if (lane == 0) ps[j * chunk + t] = a * scale;
    }
  }
  __syncthreads();
  // softmax pieces per head: one warp per head
  for (int j = wid; j < G; j += nw) {
    float m = -INFINITY;
    for (int t = lane; t < n; t += kWarp) m = fmaxf(m, ps[j * chunk + t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < n; t += kWarp) {
      const float e = expf(ps[j * chunk + t] - m);
      ps[j * chunk + t] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      mls[2 * j] = m;
      mls[2 * j + 1] = l;
    }
  }
  __syncthreads();
  const size_t pbase = ((size_t)g * kAttnMaxSplits + s) * G;
  for (int idx = threadIdx.x; idx < G * hd; idx += blockDim.x) {
    const int j = idx / hd, e = idx - j * hd;
    float a = 0.f;
    for (int t = 0; t < n; ++t) a = fmaf(ps[j * chunk + t], vbase[(size_t)t * hd + e], a);
    part_o[(pbase + j) * hd + e] = a;
  }
  if (threadIdx.x < G) {
    part_ml[(pbase + threadIdx.x) * 2] = mls[2 * threadIdx.x];
    part_ml[(pbase + threadIdx.x) * 2 + 1] = mls[2 * threadIdx.x + 1];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = (atomicAdd(cnt + g, 1u) == (unsigned)nsplit - 1u);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int idx = threadIdx.x; idx < G * hd; idx += blockDim.x) {
    const int j = idx / hd, e = idx - j * hd;
    float M = -INFINITY;
    for (int r = 0; r < nsplit; ++r)
      M = fmaxf(M, __ldcg(part_ml + (((size_t)g * kAttnMaxSplits + r) * G + j) * 2));
    float L = 0.f, O = 0.f;
    for (int r = 0; r < nsplit; ++r) {
      const size_t pj = ((size_t)g * kAttnMaxSplits + r) * G + j;
      const float w = expf(__ldcg(part_ml + pj * 2) - M);
      L += __ldcg(part_ml + pj * 2 + 1) * w;
      O += __ldcg(part_o + pj * hd + e) * w;
    }
    const float inv = 1.0f / (L + 1e-12f);
    out[((size_t)g * G + j) * hd + e] = O * inv;
  }
  if (threadIdx.x == 0) cnt[g] = 0u;  // ready for the next launch
}

__global__ void __launch_bounds__(kAttnThreads) k_attn(StepParams P, LayerW W) {
  const int ctx = (int)P.st->pos + 1;
  attn_core(P.q, W.kc, W.vc, P.attn, ctx, P.max_ctx, P.nh, P.nkv, P.hd, P.attn_scale, P.part_o,
            P.part_ml, P.attn_cnt);
}

// attn_output GEMV + residual: x[n] = x[n] + y[n].
__global__ void __launch_bounds__(kGemvThreads) k_oproj(StepParams P, LayerW W) {
  extern __shared__ float smem[];
  float* xs = smem;  // [nh*hd] swizzled
  const int K = W.wo.K;
  for (int i = threadIdx.x; i < K; i += blockDim.x) xs[swz(i)] = P.attn[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int r = gw; r < W.wo.N; r += nwarps) {
    const float y = q4_row(W.wo, r, xs, lane);
    if (lane == 0) P.x[r] = P.x[r] + y;
  }
}

// SwiGLU of activation.rs:35-51 (swiglu_balanced).
__device__ __forceinline__ float swiglu_balanced(float g, float u) {
  const float gs = rclamp(g, -64.0f, 64.0f);
  float sig;
  if (gs >= 0.0f) {
    sig = 1.0f / (1.0f + expf(-gs));
  } else {
    const float ex = expf(gs);
    sig = ex / (1.0f + ex);
  }
  return (g * sig) * u;
}

// ffn_norm prologue + ffn_gate_up GEMV (rows n and ff+n per warp) + SwiGLU.
__global__ void __launch_bounds__(kGemvThreads) k_gateup(StepParams P, LayerW W, int layer) {
  extern __shared__ float smem[];
  float* xs = smem;  // [d] swizzled
  __shared__ float red[32];
  bool nan_in, nan_out;
  rmsnorm_smem(P.x, W.ffn_norm, P.eps, P.d, xs, red, nan_in, nan_out);
  const int lane = threadIdx.x & 31;
  const int ff = W.gate_up.N >> 1;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int n = gw; n < ff; n += nwarps) {
    float g, u;
    q4_row2(W.gate_up, n, n + ff, xs, lane, g, u);
    if (lane == 0) {
      if (u != u) nan_flag(P.st, layer, kNanUp);
      const float a = swiglu_balanced(g, u);
      if (a != a) nan_flag(P.st, layer, kNanFfnOut);
      P.act[n] = a;
    }
  }
}

// ffn_down GEMV + residual.  With use_genomic_norm (block/forward.rs:115-123)
// every CTA first rescales act by h_scale/rms when rms > h_scale (h_scale = 1).
__global__ void __launch_bounds__(kGemvThreads) k_down(StepParams P, LayerW W, int layer) {
  extern __shared__ float smem[];
  float* xs = smem;  // [ff] swizzled
  __shared__ float red[32];
  const int K = W.down.K;
  float s = 1.0f;
  if (P.use_genomic_norm) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < K; i += blockDim.x) ss = fmaf(P.act[i], P.act[i], ss);
    ss = block_sum(ss, red);
    const float rms = sqrtf(ss / (float)K + P.eps);
    if (rms > 1.0f) s = 1.0f / rms;
  }
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    const float a = P.act[i];
    xs[swz(i)] = P.use_genomic_norm && s != 1.0f ? a * s : a;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int r = gw; r < W.down.N; r += nwarps) {
    const float y = q4_row(W.down, r, xs, lane);
    if (lane == 0) {
      if (y != y) nan_flag(P.st, layer, kNanProjFfn);
      const float xn = P.x[r] + y;
      if (xn != xn) nan_flag(P.st, layer, kNanResidual);
      P.x[r] = xn;
    }
  }
}

// Orderable key for the first-max argmax: larger value wins, then the lower
// index.  NaN and -inf never win (the reference's strict `val > max_val`
// against a -inf start, llm/forward.rs:262-271); -0.0 ties with +0.0.
__device__ __forceinline__ unsigned long long amax_key(float v, unsigned idx) {
  if (!(v > -INFINITY)) return 0ull;
  if (v == 0.0f) v = 0.0f;
  unsigned u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (0xFFFFFFFFu - idx);
}
__host__ __device__ __forceinline__ unsigned amax_index(unsigned long long key) {
  return key ? 0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull) : 0u;
}

// Final-CTA argmax reduction shared by the lm_head kernels.
__device__ __forceinline__ void amax_finish(unsigned long long best, unsigned long long* part,
                                            unsigned* cnt, unsigned* result, StepParams* P) {
  __shared__ unsigned long long wbest[32];
  __shared__ int is_last;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  best = warp_max_u64(best);
  if (lane == 0) wbest[wid] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0;
    for (int i = 0; i < nw; ++i) b = wbest[i] > b ? wbest[i] : b;
    part[blockIdx.x] = b;
    __threadfence();
    is_last = (atomicAdd(cnt, 1u) == gridDim.x - 1u);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  unsigned long long b = 0;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) {
    const unsigned long long v = __ldcg(part + i);
    b = v > b ? v : b;
  }
  b = warp_max_u64(b);
  __syncthreads();
  if (lane == 0) wbest[wid] = b;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long r = 0;
    for (int i = 0; i < nw; ++i) r = wbest[i] > r ? wbest[i] : r;
    const unsigned idx = amax_index(r);
    *result = idx;
    *cnt = 0u;
    if (P) {  // advance the decode state
      DevState* st = P->st;
      st->argmax = idx;
      st->token = idx;
      if (st->hist_len < P->hist_cap) P->tok_hist[st->hist_len] = idx;
      st->hist_len += 1u;
      st->pos += 1u;
    }
  }
}

// FP32 GEMV core: warp per row, float4 loads with an evict-first hint (the
// matrix is streamed once per step), x from smem.  Requires K % 4 == 0.
__device__ __forceinline__ unsigned long long f32_rows(const float* __restrict__ W,
                                                       const float* __restrict__ bias,
                                                       const float* xs, int N, int K,
                                                       float* __restrict__ logits) {
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const int K4 = K >> 2;
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  unsigned long long best = 0ull;
  int r = gw;
  for (; r + nwarps < N; r += 2 * nwarps) {
    const float4* w0 = reinterpret_cast<const float4*>(W + (size_t)r * K);
    const float4* w1 = reinterpret_cast<const float4*>(W + (size_t)(r + nwarps) * K);
    float a = 0.f, c = 0.f;
#pragma unroll 4
    for (int j = lane; j < K4; j += kWarp) {
      const float4 u = __ldcs(w0 + j), v = __ldcs(w1 + j), xv = x4[j];
      a = fmaf(u.x, xv.x, a); a = fmaf(u.y, xv.y, a); a = fmaf(u.z, xv.z, a); a = fmaf(u.w, xv.w, a);
      c = fmaf(v.x, xv.x, c); c = fmaf(v.y, xv.y, c); c = fmaf(v.z, xv.z, c); c = fmaf(v.w, xv.w, c);
    }
    a = warp_sum(a);
    c = warp_sum(c);
    if (bias) { a += bias[r]; c += bias[r + nwarps]; }
    if (lane == 0 && logits) { logits[r] = a; logits[r + nwarps] = c; }
    const unsigned long long ka = amax_key(a, r), kc = amax_key(c, r + nwarps);
    best = ka > best ? ka : best;
    best = kc > best ? kc : best;
  }
  for (; r < N; r += nwarps) {
    const float4* w0 = reinterpret_cast<const float4*>(W + (size_t)r * K);
    float a = 0.f;
    for (int j = lane; j < K4; j += kWarp) {
      const float4 u = __ldcs(w0 + j), xv = x4[j];
      a = fmaf(u.x, xv.x, a); a = fmaf(u.y, xv.y, a); a = fmaf(u.z, xv.z, a); a = fmaf(u.w, xv.w, a);
    }
    a = warp_sum(a);
    if (bias) a += bias[r];
    if (lane == 0 && logits) logits[r] = a;
    const unsigned long long ka = amax_key(a, r);
    best = ka > best ? ka : best;
  }
  return best;
}

// Final RMSNorm + lm_head + argmax, advancing the decode state.
__global__ void __launch_bounds__(kLmThreads) k_lmhead(StepParams P) {
  extern __shared__ float smem[];
  float* xs = smem;  // [d] plain layout
  __shared__ float red[32];
  float ss = 0.f;
  for (int i = threadIdx.x; i < P.d; i += blockDim.x) ss = fmaf(P.x[i], P.x[i], ss);
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)P.d + P.eps);
  for (int i = threadIdx.x; i < P.d; i += blockDim.x) xs[i] = (P.x[i] * inv) * P.out_norm[i];
  __syncthreads();
  const unsigned long long best = f32_rows(P.lm_head, P.lm_bias, xs, P.V, P.d, P.logits);
  amax_finish(best, P.amax_part, P.amax_cnt, &P.st->argmax, &P);
}

// Stand-alone FP32 GEMV + argmax (op-level entry point).
__global__ void __launch_bounds__(kLmThreads) k_f32_gemv_argmax(const float* W, const float* x, int N, int K,
                                                            float* logits, unsigned long long* part,
                                                            unsigned* cnt, unsigned* result) {
  extern __shared__ float smem[];
  for (int i = threadIdx.x; i < K; i += blockDim.x) smem[i] = x[i];
  __syncthreads();
  const unsigned long long best = f32_rows(W, nullptr, smem, N, K, logits);
  amax_finish(best, part, cnt, result, nullptr);
}

// ------------------------------------------------------------------ K-WTA
__device__ __forceinline__ unsigned ord_key(float v) {
  if (v == 0.0f) v = 0.0f;
  const unsigned u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord_val(unsigned k) {
  const unsigned u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

// lateral_inhibition_kwta (lut.rs:45-61) in one CTA: an MSB-first radix select
// (4 passes of 8 bits) finds the exact k-th largest value; then every value
// strictly below it becomes -1e9.  The threshold is exact, so the mask equals
// the reference's full-sort result (NaN ordering aside).
__global__ void __launch_bounds__(kKwtaThreads) k_kwta(float* s, int n, int k) {
  __shared__ unsigned hist[256];
  __shared__ unsigned sel_prefix, sel_k;
  if (n <= k || k <= 0) return;
  unsigned prefix = 0u, mask = 0u;
  unsigned kk = (unsigned)k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const unsigned key = ord_key(s[i]);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xFFu], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned acc = 0u;
      int b = 255;
      for (; b > 0; --b) {
        if (acc + hist[b] >= kk) break;
        acc += hist[b];
      }
      sel_prefix = prefix | ((unsigned)b << shift);
      sel_k = kk - acc;
    }
    __syncthreads();
    prefix = sel_prefix;
    kk = sel_k;
    mask |= 0xFFu << shift;
    __syncthreads();
  }
  const float thr = ord_val(prefix);
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    if (s[i] < thr) s[i] = -1e9f;
}

// ---------------------------------------------------------- setup kernels
// File blocks (20 bytes, 4-byte aligned) -> qs/sm arrays, row offset `row0`.
__global__ void k_repack_q4(const uint32_t* __restrict__ raw, size_t nblocks, uint4* qs, uint32_t* sm) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nblocks;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t* b = raw + i * 5;
    sm[i] = b[0];
    qs[i] = make_uint4(b[1], b[2], b[3], b[4]);
  }
}

// Bit-exact dequantisation: w = fmaf(q, scale, min) (genomic.rs:298).
__global__ void k_dequant_q4(Q4View W, float* out) {
  const size_t total = (size_t)W.N * W.K;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / W.K;
    const int col = (int)(i - row * W.K);
    const int b = col >> 5, e = col & 31;
    const uint4 q = W.qs[row * W.nb + b];
    const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
    float scale, mn;
    unpack_sm(W.sm[row * W.nb + b], scale, mn);
    const uint32_t word = wd[e >> 3];
    const int byte = (e & 7) >> 1;
    const uint32_t code = (word >> (8 * byte + 4 * (e & 1))) & 0xFu;
    out[i] = fmaf((float)code, scale, mn);
  }
}

// Op-level Q4_0 GEMV over M input vectors: grid (ctas, M).
__global__ void __launch_bounds__(kGemvThreads) k_q4_gemv(Q4View W, const float* x, float* y) {
  extern __shared__ float smem[];
  const float* xm = x + (size_t)blockIdx.y * W.K;
  for (int i = threadIdx.x; i < W.K; i += blockDim.x) smem[swz(i)] = xm[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int r = gw; r < W.N; r += nwarps) {
    const float v = q4_row(W, r, smem, lane);
    if (lane == 0) y[(size_t)blockIdx.y * W.N + r] = v;
  }
}

__global__ void k_rmsnorm(const float* x, const float* w, float eps, int n, float* out) {
  __shared__ float red[32];
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)n + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = (x[i] * inv) * w[i];
}

__global__ void __launch_bounds__(kAttnThreads) k_attn_op(const float* q, const float* kc, const float* vc,
                                                      float* out, int ctx, int stride, int nh, int nkv,
                                                      int hd, float scale, float* part_o, float* part_ml,
                                                      unsigned* cnt) {
  attn_core(q, kc, vc, out, ctx, stride, nh, nkv, hd, scale, part_o, part_ml, cnt);
}

}  // namespace gaje
