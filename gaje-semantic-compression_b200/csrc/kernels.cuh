// kernels.cuh -- sm_100a kernels of the batch-1 decode step.
//
// One decode step of GenomicLLM::forward_core (src/nn/llm/forward.rs:7-63) is
// five kernels per block plus the lm_head, chained with programmatic dependent
// launch (PDL):
//   k_gemv<G_QKV>     attn_norm RMSNorm (norm.rs:17-87) + Q4_0 GEMV of attn_qkv
//                     (genomic.rs:267-336 with the flush and bias of
//                     linear/forward.rs:84-115) + RoPE (attention.rs:62-84)
//                     + KV-cache append (attention.rs:85-86)
//   k_attn            split-K flash-decode GQA attention (attention.rs:88-127);
//                     the last CTA of each KV head combines the splits
//   k_gemv<G_OPROJ>   attn_output GEMV + residual (block/forward.rs:76-82)
//   k_gemv<G_GATEUP>  ffn_norm RMSNorm + ffn_gate_up GEMV + SwiGLU
//                     (activation.rs:35-51)
//   k_gemv<G_DOWN>    ffn_down GEMV + residual (block/forward.rs:124-136)
//   k_lmhead          output_norm RMSNorm + FP32 lm_head GEMV (dot.rs:46-67)
//                     + first-max argmax (llm/forward.rs:262-271)
// Optional: k_kwta (lut.rs:45-61) on the logits or on the hidden state.
//
// Data movement (B200): every CTA stages the bytes it will consume into shared
// memory with 1-D TMA bulk copies (cp.async.bulk, no multicast) completing on
// an mbarrier.  Weights and cached K/V do not depend on the previous kernel,
// so each kernel issues those copies first, then griddepcontrol.wait, then
// griddepcontrol.launch_dependents: the next kernel's copies overlap this
// kernel's math.  A kernel triggers its dependents only after its own wait,
// so when a kernel's pre-wait code runs, every kernel before its predecessor
// has completed (the decode position and earlier cache rows are stable).
// Data the immediately preceding kernel wrote is read after the wait with
// L2-only loads (ld.global.cg).
//
// Numerics: compiled with --fmad=false; every FMA is an explicit fmaf().  The
// Q4_0 dequantised weight is fmaf(q, scale, min), bit-identical to the AVX2
// kernel's fused dequant (genomic.rs:298).  Summation orders differ from the
// AVX2 8-lane order, so dot products agree to rounding, not bit for bit.
//
// Device errors are status words, never traps: NaN guards (block/forward.rs
// :11-140) record the first (position, layer, check) with atomicMin; a bounded
// mbarrier wait that runs out sets DevState::err and the kernel returns.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gaje {

constexpr int kWarp = 32;
constexpr int kGemvThreads = 512;       // 16 warps per GEMV CTA
constexpr int kAttnThreads = 256;
constexpr int kAttnMinChunk = 32;       // positions per attention split (minimum)
constexpr int kAttnMaxSplits = 64;
constexpr int kAttnMaxGroup = 16;       // q heads per kv head
constexpr int kLmConsumerWarps = 8;
constexpr int kLmThreads = (kLmConsumerWarps + 1) * 32;  // + one producer warp
constexpr int kLmRowsPerStage = 8;
constexpr int kLmMaxStages = 8;
constexpr size_t kLmSmemBudget = 200 * 1024;  // ring + x, below the 227 KB per-CTA limit
constexpr int kKwtaThreads = 1024;
constexpr int kSmemHeader = 128;        // mbarriers at the start of dynamic smem
// Limit of every bounded device-side wait (mbarrier phases, exchange flags and
// words), in ns of %globaltimer: 2 s unless gaje_cuda_set_wait_limit changed it
// for the device.
constexpr unsigned long long kWaitNsDefault = 2000000000ull;
__constant__ unsigned long long c_wait_ns = kWaitNsDefault;

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
  unsigned err;        // 0, or 1 + the kernel id of a bounded wait that ran out
  unsigned pad[2];
};

// A Q4_0 matrix in the engine's layout: per row, nb = K/32 blocks; qs[row][b]
// holds the block's 16 nibble bytes unchanged (element 2k = low nibble of
// byte k); sm[row][b] = f16 scale | f16 min << 16 with a row stride of nbp
// (nb rounded up to a multiple of 4) so that any row range is a 16-byte
// multiple for the bulk copies.  20 bytes per 32 weights, as in the file.
struct Q4View {
  const uint4* qs;
  const uint32_t* sm;
  const float* bias;  // [N] or nullptr
  int N, K, nb, nbp;
  // Genomic4Bit (genomic.rs:149-204): 16 f32 centroids per (row, block)
  // [N][nb][16]; qs then holds the codes (element 2k in the low nibble of
  // byte k, as for Q4_0) and sm is unused.  nullptr for Q4_0.
  const float* lut;
};

struct LayerW {
  Q4View qkv, wo, gate_up, down;  // qkv and gate_up rows are stored pair-interleaved
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
  int lm_flush;          // 1: the |t| < 1e-6 -> 0 flush of a Q8_0 lm_head row dot (genomic.rs:444-448)
  const unsigned char* lm_q8;  // Q8_0 lm_head rows [V][lm_row_bytes] (int8[d], f16[d/32], pad) or nullptr
  int lm_row_bytes;      // bytes of one streamed lm_head row: d*4 (f32) or the Q8_0 row above
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

// ------------------------------------------------------------------ PTX
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Makes mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait on an mbarrier phase: false after c_wait_ns without completion.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > c_wait_ns) return false;
  return true;
}
// An L2 cache policy for the cache-hinted copy below: lines loaded under it
// are the first to be evicted (data read once).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// 1-D TMA bulk copy global -> this CTA's shared memory with an L2 cache
// policy (no multicast).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
// 1-D TMA bulk copy global -> this CTA's shared memory (no multicast).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Per-thread asynchronous global -> shared copies (16 B bypassing L1, 4 B),
// tracked by an mbarrier: the arrival counts as one of the barrier's expected
// arrivals (.noinc) and fires when this thread's earlier copies have landed.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Records a timed-out wait (kernel id), keeping the first one.
__device__ __forceinline__ void flag_timeout(DevState* st, unsigned kid) { atomicCAS(&st->err, 0u, 1u + kid); }

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

// Row dot of one Q4_0 row held in shared memory (qs_row[nb], sm_row[nb]), one
// warp, lanes striding the blocks; flushed like compute_single_row (no bias).
__device__ __forceinline__ float q4_row_smem(const uint4* qs_row, const uint32_t* sm_row, int nb,
                                             const float* xs, int lane) {
  float acc = 0.f;
  for (int b = lane; b < nb; b += kWarp) acc += q4_block_dot(qs_row[b], sm_row[b], xs, b);
  return flush_small(warp_sum(acc));
}

// Genomic4Bit row dot (genomic.rs:149-204: sum of c[code] * x, each product
// rounded then added, |t| < 1e-6 flushed) from staged codes and centroid
// tables: lane l takes element l of every block, so the 32 lanes read one
// block's 64-byte table (no bank conflicts) and its 32 consecutive x.
__device__ __forceinline__ float lut4_row_smem(const uint4* qs_row, const float* lut_row, int nb, const float* xs,
                                              int lane) {
  const unsigned char* codes = reinterpret_cast<const unsigned char*>(qs_row);
  float acc = 0.f;
#pragma unroll 4
  for (int b = 0; b < nb; ++b) {
    const unsigned code = (codes[b * 16 + (lane >> 1)] >> ((lane & 1) * 4)) & 0xFu;
    acc = __fadd_rn(acc, __fmul_rn(lut_row[b * 16 + code], xs[swz((b << 5) + lane)]));
  }
  return flush_small(warp_sum(acc));
}

// Row dot straight from global memory (op-level M > 1 path).
__device__ __forceinline__ float q4_row_global(const Q4View& W, int row, const float* xs, int lane) {
  const uint4* qs = W.qs + (size_t)row * W.nb;
  const uint32_t* sm = W.sm + (size_t)row * W.nbp;
  float acc = 0.f;
#pragma unroll 4
  for (int b = lane; b < W.nb; b += kWarp) acc += q4_block_dot(__ldg(qs + b), __ldg(sm + b), xs, b);
  float y = flush_small(warp_sum(acc));
  if (W.bias) y += __ldg(W.bias + row);
  return y;
}

// NaN guard code: position * 4096 + layer * 8 + check, so atomicMin keeps the
// first failing check of the first failing step, the one the reference stops at.
__device__ __forceinline__ void nan_flag(DevState* st, unsigned pos, int layer, unsigned check) {
  atomicMin(&st->nan_code, pos * 4096u + unsigned(layer) * 8u + check);
}

// SwiGLU of activation.rs:35-51 (swiglu_balanced): sigma = 1 / (1 + e^-g) for
// g >= 0, e^g / (1 + e^g) below, on the clamped g.  Both arms take the same
// exponential, e^-|g|, so one expf, one select and one division give the two
// arms' values exactly, without divergent branches.
__device__ __forceinline__ float swiglu_balanced(float g, float u) {
  const float gs = rclamp(g, -64.0f, 64.0f);
  const float ex = expf(-fabsf(gs));
  const float sig = (gs >= 0.0f ? 1.0f : ex) / (1.0f + ex);
  return (g * sig) * u;
}

// ------------------------------------------------------------ Q4_0 GEMV
enum GemvMode { G_QKV = 0, G_OPROJ = 1, G_GATEUP = 2, G_DOWN = 3, G_PLAIN = 4 };

struct GemvArgs {
  Q4View W;
  int units;      // work units: rows (OPROJ, DOWN, PLAIN) or row pairs (QKV, GATEUP)
  int upc;        // units per CTA
  const float* x; // PLAIN: input vector
  float* y;       // PLAIN: output vector
  int layer;
};

__host__ __device__ constexpr int gemv_rows_per_unit(int mode) { return (mode == G_QKV || mode == G_GATEUP) ? 2 : 1; }

// Dynamic shared memory of a GEMV CTA: header + x (K floats) + staged rows
// (Q4_0 codes and scale/min words, or Genomic4Bit codes and centroid tables).
__host__ __device__ inline size_t gemv_smem_bytes(int mode, int K, int nb, int nbp, int upc, bool lut = false) {
  const size_t rows = size_t(upc) * gemv_rows_per_unit(mode);
  return kSmemHeader + size_t(K) * 4 + rows * nb * 16 + (lut ? rows * nb * 64 : rows * nbp * 4);
}

// One CTA owns units [u0, u1) = a contiguous row range of the (pair-
// interleaved) matrix, staged into shared memory by two bulk copies.
template <int MODE>
__global__ void __launch_bounds__(kGemvThreads) k_gemv(StepParams P, LayerW L, GemvArgs A) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw);
  __shared__ float red[32];
  constexpr int RPU = gemv_rows_per_unit(MODE);
  const Q4View& W = A.W;
  const int K = W.K, nb = W.nb, nbp = W.nbp;
  float* xs = reinterpret_cast<float*>(smem_raw + kSmemHeader);
  uint4* qs_s = reinterpret_cast<uint4*>(xs + K);
  const int u0 = blockIdx.x * A.upc;
  const int u1 = min(A.units, u0 + A.upc);
  const int r0 = u0 * RPU, nrows = (u1 - u0) * RPU;
  uint32_t* sm_s = reinterpret_cast<uint32_t*>(qs_s + (size_t)A.upc * RPU * nb);
  float* lut_s = reinterpret_cast<float*>(sm_s);  // Genomic4Bit: the centroid tables in place of sm

  // 1. stage this CTA's weight rows (independent of the previous kernel)
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t qb = uint32_t(nrows) * nb * 16;
    const uint32_t sb = W.lut ? uint32_t(nrows) * nb * 64 : uint32_t(nrows) * nbp * 4;
    mbar_expect_tx(bar, qb + sb);
    bulk_g2s(qs_s, W.qs + (size_t)r0 * nb, qb, bar);
    if (W.lut) bulk_g2s(lut_s, W.lut + (size_t)r0 * nb * 16, sb, bar);
    else bulk_g2s(sm_s, W.sm + (size_t)r0 * nbp, sb, bar);
  }
  // 2. wait for the previous kernel, release the next one
  pdl_wait();
  pdl_trigger();
  DevState* st = P.st;
  const unsigned pos = __ldcg(&st->pos);

  // 3. activation vector -> swizzled smem (RMSNorm where the reference has one)
  if (MODE == G_QKV || MODE == G_GATEUP) {
    const float* src = P.x;
    const float* nw = MODE == G_QKV ? L.attn_norm : L.ffn_norm;
    if (MODE == G_QKV && A.layer == 0) {
      const unsigned tok = __ldcg(&st->token) % (unsigned)P.V;
      src = P.embd + (size_t)tok * P.d;  // get_row_core: row token % V
    }
    float ss = 0.f;
    int bad = 0;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
      const float v = __ldcg(src + i);
      xs[swz(i)] = v;
      ss = fmaf(v, v, ss);
      bad |= (v != v);
    }
    ss = block_sum(ss, red);
    const int bad_in = __syncthreads_or(bad);
    const float inv = 1.0f / sqrtf(ss / (float)K + P.eps);
    int bad_out = 0;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
      const int si = swz(i);
      const float o = (xs[si] * inv) * nw[i];
      bad_out |= (o != o);
      xs[si] = o;
    }
    bad_out = __syncthreads_or(bad_out);
    if (MODE == G_QKV && blockIdx.x == 0) {
      if (threadIdx.x == 0) {
        if (bad_in) nan_flag(st, pos, A.layer, kNanInput);
        if (bad_out) nan_flag(st, pos, A.layer, kNanAttnNorm);
      }
      if (A.layer == 0)  // the residual stream starts as the embedding row
        for (int i = threadIdx.x; i < K; i += blockDim.x) P.x[i] = __ldcg(src + i);
    }
  } else {
    const float* src = MODE == G_OPROJ ? P.attn : (MODE == G_DOWN ? P.act : A.x);
    float s = 1.0f;
    if (MODE == G_DOWN && P.use_genomic_norm) {  // block/forward.rs:115-123, h_scale = 1
      float ss = 0.f;
      for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const float v = __ldcg(src + i);
        ss = fmaf(v, v, ss);
      }
      ss = block_sum(ss, red);
      const float rms = sqrtf(ss / (float)K + P.eps);
      if (rms > 1.0f) s = 1.0f / rms;
    }
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
      const float v = __ldcg(src + i);
      xs[swz(i)] = (s != 1.0f) ? v * s : v;
    }
    __syncthreads();
  }

  // 4. weights staged?
  if (!mbar_wait(bar, 0)) {
    if (threadIdx.x == 0) flag_timeout(st, MODE);
    mbar_wait(bar, 0);  // do not free smem under an in-flight copy (bounded again)
    return;
  }

  // 5. one warp per unit
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int u = u0 + wid; u < u1; u += nwarps) {
    const int lr = (u - u0) * RPU;
    if (RPU == 1) {
      float y = W.lut ? lut4_row_smem(qs_s + (size_t)lr * nb, lut_s + (size_t)lr * nb * 16, nb, xs, lane)
                      : q4_row_smem(qs_s + (size_t)lr * nb, sm_s + (size_t)lr * nbp, nb, xs, lane);
      if (lane == 0) {
        const int r = r0 + lr;
        if (W.bias) y += W.bias[r];
        if (MODE == G_PLAIN) {
          A.y[r] = y;
        } else if (MODE == G_OPROJ) {
          P.x[r] = __ldcg(P.x + r) + y;
        } else {  // G_DOWN
          if (y != y) nan_flag(st, pos, A.layer, kNanProjFfn);
          const float xn = __ldcg(P.x + r) + y;
          if (xn != xn) nan_flag(st, pos, A.layer, kNanResidual);
          P.x[r] = xn;
        }
      }
    } else {
      float y0, y1;
      if (W.lut) {
        y0 = lut4_row_smem(qs_s + (size_t)lr * nb, lut_s + (size_t)lr * nb * 16, nb, xs, lane);
        y1 = lut4_row_smem(qs_s + (size_t)(lr + 1) * nb, lut_s + (size_t)(lr + 1) * nb * 16, nb, xs, lane);
      } else {
        y0 = q4_row_smem(qs_s + (size_t)lr * nb, sm_s + (size_t)lr * nbp, nb, xs, lane);
        y1 = q4_row_smem(qs_s + (size_t)(lr + 1) * nb, sm_s + (size_t)(lr + 1) * nbp, nb, xs, lane);
      }
      if (lane == 0) {
        if (W.bias) {
          y0 += W.bias[r0 + lr];
          y1 += W.bias[r0 + lr + 1];
        }
        if (MODE == G_GATEUP) {
          if (y1 != y1) nan_flag(st, pos, A.layer, kNanUp);
          const float a = swiglu_balanced(y0, y1);
          if (a != a) nan_flag(st, pos, A.layer, kNanFfnOut);
          P.act[u] = a;
        } else {  // G_QKV: pair u = (head, i) in the interleaved row order
          const int half = P.hd >> 1;
          const int head = u / half, i = u - head * half;
          const int c0 = P.rope_split ? i : 2 * i;
          const int c1 = P.rope_split ? i + half : 2 * i + 1;
          if (head < P.nh + P.nkv) {  // RoPE on q and k: v0*cos - v1*sin, v0*sin + v1*cos
            const float2 cs = P.rope[(size_t)pos * half + i];
            const float o0 = y0 * cs.x - y1 * cs.y;
            const float o1 = y0 * cs.y + y1 * cs.x;
            y0 = o0;
            y1 = o1;
          }
          if (head < P.nh) {
            P.q[head * P.hd + c0] = y0;
            P.q[head * P.hd + c1] = y1;
          } else {
            const bool is_k = head < P.nh + P.nkv;
            const int g = is_k ? head - P.nh : head - P.nh - P.nkv;
            float* c = (is_k ? L.kc : L.vc) + ((size_t)g * P.max_ctx + pos) * P.hd;
            c[c0] = y0;
            c[c1] = y1;
          }
        }
      }
    }
  }
}

// ------------------------------------------------------------ attention
// Split bookkeeping shared by the attention kernels and the host.
__host__ __device__ __forceinline__ void attn_splits(int ctx, int& nsplit, int& chunk,
                                                     int max_splits = kAttnMaxSplits) {
  int n0 = (ctx + kAttnMinChunk - 1) / kAttnMinChunk;
  if (n0 > max_splits) n0 = max_splits;
  if (n0 < 1) n0 = 1;
  chunk = (ctx + n0 - 1) / n0;
  nsplit = (ctx + chunk - 1) / chunk;
}
__host__ __device__ inline int attn_chunk_max(int max_ctx, int max_splits = kAttnMaxSplits) {
  const int c = (max_ctx + max_splits - 1) / max_splits;
  return c > kAttnMinChunk ? c : kAttnMinChunk;
}
__host__ __device__ inline size_t attn_smem_bytes(int G, int hd, int chunk_max) {
  return kSmemHeader + size_t(2 * chunk_max * hd + G * hd + G * chunk_max) * 4;
}

struct AttnArgs {
  const float* q;   // [nh*hd]
  const float* kc;  // [nkv][stride][hd]
  const float* vc;
  float* out;       // [nh*hd]
  float* part_o;
  float* part_ml;
  unsigned* cnt;    // [nkv]
  unsigned* bad;    // [nkv] or nullptr: a split of the group timed out (its output becomes NaN)
  int ctx;          // >0: fixed context (op level); 0: st->pos + 1
  int stride, nh, nkv, hd;
  float scale;
  DevState* st;     // decode state (step) or nullptr (op level)
  int fresh;        // with ctx > 0: row ctx-1 is written by the preceding kernel (batched steps)
  int max_splits;   // 0: kAttnMaxSplits (the launch's grid.y must cover the splits)
};

// One CTA per (kv head g, split s).  The split's cached K/V rows (positions
// before the new one) are bulk-copied to smem before the PDL wait; the new
// row and q are read after it.  Scores for the G query heads of the group,
// exp against the split max, unnormalised P*V; the last CTA of the group
// combines the splits:
//   out = (sum_s O_s e^{m_s-M}) * (1/(sum_s l_s e^{m_s-M} + 1e-12))
// (the reference's inv_s = 1/(sum_e + 1e-12), attention.rs:110).
__device__ __forceinline__ void attn_split(const AttnArgs& A, const int g, const int s) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw);
  __shared__ float mls[2 * kAttnMaxGroup];
  __shared__ float wsh[kAttnMaxGroup * kAttnMaxSplits];
  __shared__ float linv[kAttnMaxGroup];
  __shared__ int is_last;
  const int G = A.nh / A.nkv, hd = A.hd;
  // the decode position is stable here (written two or more kernels back)
  const int ctx = A.ctx > 0 ? A.ctx : (int)__ldcg(&A.st->pos) + 1;
  int nsplit, chunk;
  attn_splits(ctx, nsplit, chunk, A.max_splits > 0 ? A.max_splits : kAttnMaxSplits);
  if (s >= nsplit) return;
  const int t0 = s * chunk;
  const int n = min(ctx, t0 + chunk) - t0;
  // rows already in the cache before this step; the step's own row (ctx-1)
  // is written by the preceding kernel
  const int newest = (A.ctx > 0 && !A.fresh) ? ctx : ctx - 1;
  const int n_old = max(0, min(n, newest - t0));
  const int cm = chunk;  // smem row capacity used by this launch
  float* Ks = reinterpret_cast<float*>(smem_raw + kSmemHeader);
  float* Vs = Ks + (size_t)cm * hd;
  float* qs = Vs + (size_t)cm * hd;
  float* ps = qs + (size_t)G * hd;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const float* kbase = A.kc + ((size_t)g * A.stride + t0) * hd;
  const float* vbase = A.vc + ((size_t)g * A.stride + t0) * hd;
  if (threadIdx.x == 0) {
    const uint32_t bytes = uint32_t(n_old) * hd * 4;
    mbar_expect_tx(bar, 2 * bytes);
    if (bytes) {
      bulk_g2s(Ks, kbase, bytes, bar);
      bulk_g2s(Vs, vbase, bytes, bar);
    }
  }
  pdl_wait();
  pdl_trigger();
  for (int i = threadIdx.x; i < G * hd; i += blockDim.x) qs[i] = __ldcg(A.q + (size_t)g * G * hd + i);
  for (int i = threadIdx.x; i < (n - n_old) * hd; i += blockDim.x) {  // the new row
    Ks[(size_t)n_old * hd + i] = __ldcg(kbase + (size_t)n_old * hd + i);
    Vs[(size_t)n_old * hd + i] = __ldcg(vbase + (size_t)n_old * hd + i);
  }
  // a wait that ran out still arrives on the group's counter below, so the
  // counter cannot stay at a partial count; the group's output becomes NaN
  const bool ok = __syncthreads_and(mbar_wait(bar, 0)) != 0;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const size_t pbase = ((size_t)g * kAttnMaxSplits + s) * G;
  // one split: the combine below reduces to O * (1/(l + 1e-12)), written here
  const bool single = nsplit == 1;
  if (!ok) {
    if (threadIdx.x == 0 && A.st) flag_timeout(A.st, 8);
    mbar_wait(bar, 0);  // the copies land before the CTA leaves (bounded again)
    if (single) {
      for (int i = threadIdx.x; i < G * hd; i += blockDim.x) A.out[(size_t)g * G * hd + i] = __int_as_float(0x7fc00000);
      return;
    }
    if (threadIdx.x == 0 && A.bad) atomicExch(A.bad + g, 1u);
  } else {
  // scores: thread per (head j, position t); the (e + t) % hd walk keeps the
  // 32 positions of a warp on 32 different banks
  for (int idx = threadIdx.x; idx < G * n; idx += blockDim.x) {
    const int j = idx / n, t = idx - j * n;
    const float* qr = qs + j * hd;
    const float* kr = Ks + (size_t)t * hd;
    float a0 = 0.f, a1 = 0.f;
    int e0 = (t % hd) & ~1;  // head_dim is even, so e0 + 1 never wraps past hd
    for (int e = 0; e < hd; e += 2) {
      a0 = fmaf(qr[e0], kr[e0], a0);
      a1 = fmaf(qr[e0 + 1], kr[e0 + 1], a1);
      e0 += 2;
      if (e0 >= hd) e0 -= hd;
    }
    ps[j * cm + t] = (a0 + a1) * A.scale;
  }
  __syncthreads();
  for (int j = wid; j < G; j += nw) {
    float m = -INFINITY;
    for (int t = lane; t < n; t += kWarp) m = fmaxf(m, ps[j * cm + t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < n; t += kWarp) {
      const float e = expf(ps[j * cm + t] - m);
      ps[j * cm + t] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      mls[2 * j] = m;
      mls[2 * j + 1] = l;
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * hd; idx += blockDim.x) {
    const int j = idx / hd, e = idx - j * hd;
    const float* pr = ps + j * cm;
    float a0 = 0.f, a1 = 0.f;
    int t = 0;
    for (; t + 1 < n; t += 2) {
      a0 = fmaf(pr[t], Vs[(size_t)t * hd + e], a0);
      a1 = fmaf(pr[t + 1], Vs[(size_t)(t + 1) * hd + e], a1);
    }
    if (t < n) a0 = fmaf(pr[t], Vs[(size_t)t * hd + e], a0);
    if (single) A.out[((size_t)g * G + j) * hd + e] = (a0 + a1) * (1.0f / (mls[2 * j + 1] + 1e-12f));
    else A.part_o[(pbase + j) * hd + e] = a0 + a1;
  }
  if (single) return;
  if (threadIdx.x < G) {
    A.part_ml[(pbase + threadIdx.x) * 2] = mls[2 * threadIdx.x];
    A.part_ml[(pbase + threadIdx.x) * 2 + 1] = mls[2 * threadIdx.x + 1];
  }
  }  // ok
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = (atomicAdd(A.cnt + g, 1u) == (unsigned)nsplit - 1u);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (A.bad && __ldcg(A.bad + g)) {  // a split of the group gave up: no valid partials
    for (int i = threadIdx.x; i < G * hd; i += blockDim.x) A.out[(size_t)g * G * hd + i] = __int_as_float(0x7fc00000);
    __syncthreads();
    if (threadIdx.x == 0) {
      A.bad[g] = 0u;
      A.cnt[g] = 0u;
    }
    return;
  }
  // combine: per-split weights w = e^{m_s - M} in smem, then O in parallel
  for (int idx = threadIdx.x; idx < G * nsplit; idx += blockDim.x) {
    const int j = idx / nsplit, r = idx - j * nsplit;
    wsh[idx] = __ldcg(A.part_ml + (((size_t)g * kAttnMaxSplits + r) * G + j) * 2);
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
      Lsum += __ldcg(A.part_ml + (((size_t)g * kAttnMaxSplits + r) * G + j) * 2 + 1) * w;
    }
    Lsum = warp_sum(Lsum);
    if (lane == 0) linv[j] = 1.0f / (Lsum + 1e-12f);
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * hd; idx += blockDim.x) {
    const int j = idx / hd, e = idx - j * hd;
    const float* po = A.part_o + ((size_t)g * kAttnMaxSplits * G + j) * hd + e;  // split r at + r*G*hd
    float O0 = 0.f, O1 = 0.f;
    for (int r0 = 0; r0 < nsplit; r0 += 8) {  // eight partials in flight per thread
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = r0 + k < nsplit ? __ldcg(po + (size_t)(r0 + k) * G * hd) : 0.f;
#pragma unroll
      for (int k = 0; k < 8; k += 2) {
        if (r0 + k < nsplit) O0 += v[k] * wsh[j * nsplit + r0 + k];
        if (r0 + k + 1 < nsplit) O1 += v[k + 1] * wsh[j * nsplit + r0 + k + 1];
      }
    }
    A.out[((size_t)g * G + j) * hd + e] = (O0 + O1) * linv[j];
  }
  if (threadIdx.x == 0) A.cnt[g] = 0u;  // ready for the next launch
}
__global__ void __launch_bounds__(kAttnThreads) k_attn(AttnArgs A) { attn_split(A, blockIdx.x, blockIdx.y); }

// ------------------------------------------------------------ lm_head
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

struct LmArgs {
  const float* W;      // [N][K]
  const float* bias;   // [N] or nullptr
  const float* x;      // input (normalised unless norm_w is set)
  const float* norm_w; // final RMSNorm weight, or nullptr for a plain GEMV
  float eps;
  float* logits;       // [N] or nullptr
  int N, K, rows_per_cta, stages;
  int flush;           // 1: flush |t| < 1e-6 to 0 before the bias (a Q8_0 lm_head)
  unsigned long long* part;
  unsigned* cnt;
  unsigned* result;
  DevState* st;        // non-null: advance the decode state
  unsigned* tok_hist;
  unsigned hist_cap;
};

// Ring depth for a row length K: as many 8-row stages as fit the budget.
__host__ __device__ inline int lm_stages(int K) {
  const size_t stage = size_t(kLmRowsPerStage) * K * 4;
  const size_t avail = kLmSmemBudget - size_t(K) * 4;
  int s = int(avail / stage);
  return s > kLmMaxStages ? kLmMaxStages : s;
}
__host__ __device__ inline size_t lm_smem_bytes(int K, int stages) {
  return kSmemHeader + size_t(K) * 4 + size_t(stages) * kLmRowsPerStage * K * 4;
}

// Persistent streaming GEMV: each CTA owns a contiguous row range; a producer
// warp streams kLmRowsPerStage rows per stage into a ring of A.stages smem
// with bulk copies (full/empty mbarrier pairs), the first stages before the
// PDL wait; consumer warps compute one row each per stage from smem.
__global__ void __launch_bounds__(kLmThreads) k_lmhead(LmArgs A) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty = full + kLmMaxStages;
  const int S = A.stages;
  float* xs = reinterpret_cast<float*>(smem_raw + kSmemHeader);
  float* ring = xs + A.K;
  __shared__ float red[32];
  __shared__ unsigned long long wbest[32];
  __shared__ int is_last;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int rbeg = blockIdx.x * A.rows_per_cta;
  const int rend = min(A.N, rbeg + A.rows_per_cta);
  const int nrows = max(0, rend - rbeg);
  const int nstage = (nrows + kLmRowsPerStage - 1) / kLmRowsPerStage;
  const size_t stage_floats = size_t(kLmRowsPerStage) * A.K;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, kLmConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  unsigned long long best = 0ull;
  bool timed_out = false;
  if (wid == kLmConsumerWarps) {
    // ---------------- producer warp
    if (lane == 0) {
      for (int k = 0; k < nstage; ++k) {
        const int slot = k % S;
        if (k >= S && !mbar_wait(empty + slot, ((k / S) - 1) & 1)) {
          timed_out = true;
          break;
        }
        const int row = rbeg + k * kLmRowsPerStage;
        const int rows = min(kLmRowsPerStage, rend - row);
        const uint32_t bytes = uint32_t(rows) * A.K * 4;
        mbar_expect_tx(full + slot, bytes);
        bulk_g2s(ring + slot * stage_floats, A.W + (size_t)row * A.K, bytes, full + slot);
      }
    }
    pdl_wait();
    pdl_trigger();
  } else {
    // ---------------- consumer warps
    pdl_wait();
    pdl_trigger();
    const int cthreads = kLmConsumerWarps * 32;
    if (A.norm_w) {  // output_norm RMSNorm (llm/forward.rs:28)
      float ss = 0.f;
      for (int i = threadIdx.x; i < A.K; i += cthreads) {
        const float v = __ldcg(A.x + i);
        xs[i] = v;
        ss = fmaf(v, v, ss);
      }
      ss = warp_sum(ss);
      if (lane == 0) red[wid] = ss;
      asm volatile("bar.sync 1, %0;" ::"r"(cthreads));
      float t = lane < kLmConsumerWarps ? red[lane] : 0.f;
      t = warp_sum(t);
      const float inv = 1.0f / sqrtf(t / (float)A.K + A.eps);
      for (int i = threadIdx.x; i < A.K; i += cthreads) xs[i] = (xs[i] * inv) * A.norm_w[i];
    } else {
      for (int i = threadIdx.x; i < A.K; i += cthreads) xs[i] = __ldcg(A.x + i);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(cthreads));
    const float4* x4 = reinterpret_cast<const float4*>(xs);
    const int K4 = A.K >> 2;
    for (int k = 0; k < nstage; ++k) {
      const int slot = k % S;
      if (!mbar_wait(full + slot, (k / S) & 1)) {
        timed_out = true;
        break;
      }
      const int row = rbeg + k * kLmRowsPerStage + wid;
      if (row < rend) {
        const float4* w4 = reinterpret_cast<const float4*>(ring + slot * stage_floats + (size_t)wid * A.K);
        float a0 = 0.f, a1 = 0.f;
        for (int j = lane; j < K4; j += kWarp) {
          const float4 u = w4[j], xv = x4[j];
          a0 = fmaf(u.x, xv.x, a0);
          a1 = fmaf(u.y, xv.y, a1);
          a0 = fmaf(u.z, xv.z, a0);
          a1 = fmaf(u.w, xv.w, a1);
        }
        float a = warp_sum(a0 + a1);
        if (A.flush) a = flush_small(a);
        if (A.bias) a += A.bias[row];
        if (lane == 0 && A.logits) A.logits[row] = a;
        const unsigned long long key = amax_key(a, (unsigned)row);
        best = key > best ? key : best;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + slot);
    }
  }
  if (timed_out && lane == 0 && A.st) flag_timeout(A.st, 9);
  // drain: never leave a bulk copy in flight into freed smem
  if (wid == kLmConsumerWarps && lane == 0 && timed_out) {
    for (int i = 0; i < S; ++i) mbar_wait(full + i, 0);
  }
  // ---------------- CTA argmax, then the last CTA finishes the job
  best = warp_max_u64(best);
  if (lane == 0) wbest[wid] = best;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  if (threadIdx.x == 0) {
    unsigned long long b = 0;
    for (int i = 0; i < nw; ++i) b = wbest[i] > b ? wbest[i] : b;
    A.part[blockIdx.x] = b;
    __threadfence();
    is_last = (atomicAdd(A.cnt, 1u) == gridDim.x - 1u);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  unsigned long long b = 0;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) {
    const unsigned long long v = __ldcg(A.part + i);
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
    *A.result = idx;
    *A.cnt = 0u;
    if (A.st) {  // advance the decode state
      DevState* st = A.st;
      st->argmax = idx;
      st->token = idx;
      if (st->hist_len < A.hist_cap) A.tok_hist[st->hist_len] = idx;
      st->hist_len += 1u;
      st->pos += 1u;
    }
  }
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
// File blocks (20 bytes, 4-byte aligned, rows in file order) -> qs/sm arrays
// in the engine's row order: dst row r takes source row perm(r).
//   mode 0: identity
//   mode 1: attn_qkv pairs, split RoPE:       dst 2p+s <- head*hd + i + s*hd/2
//   mode 2: attn_qkv pairs, interleaved RoPE: dst 2p+s <- head*hd + 2i + s
//   mode 3: ffn_gate_up pairs:                dst 2n+s <- n + s*ff
__host__ __device__ inline int repack_src_row(int mode, int r, int hd, int ff) {
  if (mode == 0) return r;
  const int p = r >> 1, s = r & 1;
  if (mode == 3) return p + s * ff;
  const int half = hd >> 1, head = p / half, i = p - head * half;
  return mode == 1 ? head * hd + i + s * half : head * hd + 2 * i + s;
}

__global__ void k_repack_q4(const uint32_t* __restrict__ raw, int N, int nb, int nbp, int mode, int hd, int ff,
                            uint4* qs, uint32_t* sm) {
  const size_t total = (size_t)N * nb;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int r = int(i / nb), b = int(i - (size_t)r * nb);
    const uint32_t* src = raw + ((size_t)repack_src_row(mode, r, hd, ff) * nb + b) * 5;
    sm[(size_t)r * nbp + b] = src[0];
    qs[(size_t)r * nb + b] = make_uint4(src[1], src[2], src[3], src[4]);
  }
}

// Bit-exact dequantisation: w = fmaf(q, scale, min) (genomic.rs:298).
// Genomic4Bit: w = c[code] (get_row_core, linear/forward.rs:195-285).
__global__ void k_dequant_q4(Q4View W, float* out) {
  const size_t total = (size_t)W.N * W.K;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / W.K;
    const int col = (int)(i - row * W.K);
    const int b = col >> 5, e = col & 31;
    const uint4 q = W.qs[row * W.nb + b];
    const uint32_t word = (e < 8) ? q.x : (e < 16) ? q.y : (e < 24) ? q.z : q.w;
    const int byte = (e & 7) >> 1;
    const uint32_t code = (word >> (8 * byte + 4 * (e & 1))) & 0xFu;
    if (W.lut) {
      out[i] = W.lut[(row * W.nb + b) * 16 + code];
      continue;
    }
    float scale, mn;
    unpack_sm(W.sm[row * W.nbp + b], scale, mn);
    out[i] = fmaf((float)code, scale, mn);
  }
}

// Op-level Q4_0 GEMV over M > 1 input vectors: grid (ctas, M).
__global__ void __launch_bounds__(256) k_q4_gemv(Q4View W, const float* x, float* y) {
  extern __shared__ float xsm[];
  const float* xm = x + (size_t)blockIdx.y * W.K;
  for (int i = threadIdx.x; i < W.K; i += blockDim.x) xsm[swz(i)] = xm[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int r = gw; r < W.N; r += nwarps) {
    const float v = q4_row_global(W, r, xsm, lane);
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

}  // namespace gaje
