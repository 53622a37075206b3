// megakernel.cuh -- persistent batch-1 decode: every phase of every block of
// GenomicLLM::forward_core (src/nn/llm/forward.rs:7-63), for n consecutive
// greedy steps, in one cooperative launch of one CTA per SM.
//
// Phases of a step, per block l:
//   QKV     attn_norm RMSNorm + attn_qkv GEMV + RoPE        -> q, new k/v
//   ATTN    split-K flash decode; the last CTA of a KV head
//           combines the splits                              -> attention out
//   OPROJ   attn_output GEMV + residual                      -> x_a
//   GATEUP  ffn_norm RMSNorm + ffn_gate_up GEMV + SwiGLU     -> act
//   DOWN    ffn_down GEMV + residual                         -> x_b (next block's x)
// then LM: output_norm + f32 lm_head GEMV + argmax            -> next token.
//
// No grid barriers.  Every vector a phase publishes goes to global memory as
// "LL" words: 8 bytes {float bits, epoch}, written and read as one 64-bit
// access, so a reader that sees the expected epoch also has the value.  A CTA
// starts a phase as soon as the words it needs carry the phase's epoch (a
// bounded spin); the all-to-all dependencies between phases order the reuse of
// each buffer.  Data that is not LL (KV-cache rows, split partials, argmax
// partials) is ordered by release/acquire fences around the LL traffic.
//
// Warp roles: warps 0-14 compute ("consumers"); lane 0 of warp 15 is a
// producer that walks this CTA's static schedule of weight "items" (the rows
// of each GEMV phase, the lm_head row stages) and streams each item into a
// ring of shared-memory slots with 1-D TMA bulk copies (no multicast),
// full/empty mbarrier pairs per slot.  It runs up to a ring ahead of the
// consumers, so the next phases' weights are in flight while the consumers
// wait for activations.  The cached K/V rows of a CTA's attention split are
// fetched by the consumers themselves (TMA, at the start of the block's QKV
// phase), once the previous step's rows are known to be written.
//
// Q4_0 row dots (the AVX2 kernel's arithmetic, genomic.rs:267-336, factored):
// y = sum_b scale_b * A_b + min_b * X_b with A_b = sum_k q_k x_k and
// X_b = sum_k x_k.  q_k is obtained without shifting most nibbles: OR-ing the
// nibble found at bit position p of its word into the mantissa of 2^23 gives
// 2^23 + q*2^p exactly (p <= 16), and the activation is stored pre-scaled by
// 2^-p, so (f - 2^23) * x' = q * x exactly; the subtract and the FMA run as
// packed f32x2 instructions.
//
// Every wait is bounded (kWaitNs); a wait that runs out sets DevState::err,
// the CTA stops, drains its in-flight copies (bounded) and exits.
#pragma once

#include "kernels.cuh"

namespace gaje {

constexpr int kMkThreads = 512;
constexpr int kMkConsumerWarps = 15;
constexpr int kMkConsumers = kMkConsumerWarps * 32;
constexpr int kMkMaxSlots = 8;
constexpr int kMkHeader = 1024;       // mbarriers + flags
constexpr int kMkPartFloats = 1024;   // split-K partials / row sums
constexpr int kMkRound = 8;           // LL words per consumer thread per read round
constexpr int kMkMaxNormVec = 4;      // norm weights per thread (d <= 1920)
// Trace points of a phase, per CTA: 0 entry, 1 inputs arrived, 2 inputs
// staged (attention: cached K/V landed), 3 first weight slot taken
// (attention: split partials published), 4 done (outputs published).
constexpr int kMkTrace = 5;

// The vectors exchanged between phases, as {bits, epoch} words.
struct LLBufs {
  uint2* xa;    // [d] after the attention residual
  uint2* xb;    // [d] after the FFN residual (the next block's input)
  uint2* q;     // [nh*hd] rotated q
  uint2* kv;    // [2][nkv*hd] this step's k (rotated) and v rows
  uint2* attn;  // [nh*hd] attention output
  uint2* act;   // [ff] SwiGLU output
  uint2* tok;   // [1] the step's argmax (bits = token id)
};

struct MkGemv {
  int units, upc, units_per_item;
};

struct MegaPlan {
  int nslots;
  unsigned slot_bytes;
  MkGemv q, o, g, d;
  int lm_rows_per_cta, lm_stage_rows;
  int xs_floats;   // activation buffers capacity (>= max K, multiple of 32)
  int ps_floats;   // attention scores capacity (G * chunk cap)
  int attn_chunk_cap;
};

struct MegaArgs {
  StepParams P;
  const LayerW* layers;  // [n_layers], device memory
  MegaPlan plan;
  LLBufs ll;
  unsigned epoch0;       // epochs of this launch start after it
  int n_steps;
  int block_k;           // block K-WTA k (0 = off)
  unsigned long long* phase_ns;   // optional [n_steps][5*L+1] phase-done stamps (CTA 0)
  unsigned long long* trace_ns;   // optional [grid][n_steps][5*L+1][kMkTrace] (every CTA)
};

// Epoch of the words phase `ph` (0..4) of block l publishes in step s; the
// LM phase publishes as (l = L, ph = 0).
__host__ __device__ inline unsigned mk_epoch(unsigned e0, int L, int step, int l, int ph) {
  return e0 + unsigned(step) * unsigned(5 * L + 1) + unsigned(5 * l + ph) + 1u;
}

__host__ __device__ inline size_t mega_smem_bytes(const MegaPlan& p, int d, int hd) {
  const size_t xs = p.xs_floats;
  return kMkHeader + 4 * (2 * xs + xs / 32 + size_t(d + 31) / 32 * 32 + p.ps_floats +
                          size_t(2) * p.attn_chunk_cap * hd + kMkPartFloats + hd) +
         size_t(p.nslots) * p.slot_bytes;
}

struct MkShared {
  uint64_t* full;
  uint64_t* empty;
  uint64_t* kv_bar;
  volatile int* abort_flag;  // raised by the producer
  volatile int* issued;      // items the producer has issued
  volatile int* cabort;      // consumers' abort decision (written before, read after a consumer barrier)
  volatile int* kv_armed;    // uses of kv_bar armed so far (thread 0 of the consumers)
  volatile int* kv_waited;   // uses of kv_bar waited for
  float* xs;     // activations, RMSNormed where the phase has a norm, pre-scaled, swizzled
  float* xraw;   // activations as read
  float* xsum;   // per-32-block sums of the (normalised, unscaled) activations
  float* xres;   // the residual input of the block's OPROJ / DOWN
  float* ps;     // attention scores
  float* kvbuf;  // K rows [chunk cap][hd], then V rows
  float* part;   // split-K partials [512] + row sums [512]
  float2* rope;  // the RoPE row of the step's position
  unsigned char* slots;
};

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kMkConsumers) : "memory"); }
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ uint2 ld_ll(const uint2* p) {
  uint2 v;
  asm volatile("ld.relaxed.gpu.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_ll(uint2* p, float v, unsigned e) {
  asm volatile("st.relaxed.gpu.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(e) : "memory");
}

// Reads src[0..n) (LL words of epoch e) into dst[0..n) (plain layout), every
// consumer thread taking elements tid + k*480, kMkRound words in flight per
// round.  Accumulates sum(x^2) and any-NaN of this thread's elements.  Ends
// with an acquire fence.  False if a word did not arrive in time.
__device__ __forceinline__ bool ll_read(const uint2* src, int n, unsigned e, float* dst, float& ss, int& bad) {
  const int tid = threadIdx.x;
  for (int base = 0; base < n; base += kMkRound * kMkConsumers) {
    uint2 w[kMkRound];
#pragma unroll
    for (int k = 0; k < kMkRound; ++k) {
      const int i = base + tid + k * kMkConsumers;
      w[k] = i < n ? ld_ll(src + i) : make_uint2(0u, e);
    }
    unsigned long long t0 = 0;
    for (;;) {
      bool all = true;
#pragma unroll
      for (int k = 0; k < kMkRound; ++k) {
        if (w[k].y != e) {
          all = false;
          w[k] = ld_ll(src + base + tid + k * kMkConsumers);
        }
      }
      if (all) break;
      const unsigned long long t = global_ns();
      if (!t0) t0 = t;
      else if (t - t0 > kWaitNs) return false;
    }
#pragma unroll
    for (int k = 0; k < kMkRound; ++k) {
      const int i = base + tid + k * kMkConsumers;
      if (i < n) {
        const float v = __uint_as_float(w[k].x);
        dst[i] = v;
        ss = fmaf(v, v, ss);
        bad |= (v != v);
      }
    }
  }
  fence_acq_rel_gpu();
  return true;
}

// Sum over the consumer threads (result in every thread); red holds 16 floats.
__device__ __forceinline__ float consumer_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[wid] = v;
  consumer_sync();
  float t = lane < kMkConsumerWarps ? red[lane] : 0.f;
  t = warp_sum(t);
  consumer_sync();
  return t;
}
__device__ __forceinline__ int consumer_any(int v, int* redi) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = __any_sync(0xffffffffu, v != 0);
  if (lane == 0) redi[wid] = v;
  consumer_sync();
  int t = lane < kMkConsumerWarps ? redi[lane] : 0;
  t = __any_sync(0xffffffffu, t != 0);
  consumer_sync();
  return t;
}

// 2^-p for the bit position p of element k (0..7) of a word: 0,4,8,12,16,8,12,16.
__device__ __forceinline__ float nib_prescale(int k) {
  const int p = k < 5 ? 4 * k : 4 * k - 12;
  return __int_as_float((127 - p) << 23);
}

// xraw[0..K) -> xs (swizzled, scaled by `inv` and the weights in wreg when
// norm, then pre-scaled per nibble slot) and xsum (per-32-block sums of the
// unscaled values).  K is a multiple of 32; a warp covers whole blocks.
__device__ __forceinline__ void mk_stage_x(const MkShared& S, int K, const float* wreg, float inv, bool norm,
                                          int& bad_out) {
  const int tid = threadIdx.x, lane = tid & 31;
  int k = 0;
  for (int i = tid; i < K; i += kMkConsumers, ++k) {
    float v = S.xraw[i];
    if (norm) {
      v = (v * inv) * wreg[k < kMkMaxNormVec ? k : 0];
      bad_out |= (v != v);
    }
    S.xs[swz(i)] = v * nib_prescale(i & 7);
    const float bs = warp_sum(v);
    if (lane == 0) S.xsum[i >> 5] = bs;
  }
}

// Packed f32x2 helpers.
__device__ __forceinline__ unsigned long long pack2(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void unpack2(unsigned long long v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ unsigned long long fadd2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long ffma2(unsigned long long a, unsigned long long b,
                                                    unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// A = sum_k q_k x_k over one 32-weight block (pre-scaled swizzled activations).
__device__ __forceinline__ float q4_block_qx(const uint4 q, const float* xs, int b) {
  const float4* x4 = reinterpret_cast<const float4*>(xs + (b << 5));
  const int sw = b & 7;
  const uint32_t M = 0x4B000000u;
  const unsigned long long neg = pack2(-8388608.0f, -8388608.0f);
  unsigned long long acc0 = 0ull, acc1 = 0ull;  // (+0.0f, +0.0f)
  const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t a = wd[w], t = a >> 12;
    const float4 xa = x4[(2 * w) ^ sw], xb = x4[(2 * w + 1) ^ sw];
    const float f0 = __uint_as_float((a & 0xFu) | M), f1 = __uint_as_float((a & 0xF0u) | M);
    const float f2 = __uint_as_float((a & 0xF00u) | M), f3 = __uint_as_float((a & 0xF000u) | M);
    const float f4 = __uint_as_float((a & 0xF0000u) | M), f5 = __uint_as_float((t & 0xF00u) | M);
    const float f6 = __uint_as_float((t & 0xF000u) | M), f7 = __uint_as_float((t & 0xF0000u) | M);
    acc0 = ffma2(fadd2(pack2(f0, f1), neg), pack2(xa.x, xa.y), acc0);
    acc1 = ffma2(fadd2(pack2(f2, f3), neg), pack2(xa.z, xa.w), acc1);
    acc0 = ffma2(fadd2(pack2(f4, f5), neg), pack2(xb.x, xb.y), acc0);
    acc1 = ffma2(fadd2(pack2(f6, f7), neg), pack2(xb.z, xb.w), acc1);
  }
  float a0, a1, a2, a3;
  unpack2(acc0, a0, a1);
  unpack2(acc1, a2, a3);
  return (a0 + a1) + (a2 + a3);
}

// Rows [0, R) of one staged item -> rowsum[t] (flushed; bias added by the
// caller).  Warps split rows; with fewer rows than warps a row's blocks are
// split across g warps and the partials summed in a fixed order.
__device__ __forceinline__ void mk_rows(const MkShared& S, const unsigned char* slot, int R, int nb, int nbp,
                                        float* rowsum) {
  const uint4* qs = reinterpret_cast<const uint4*>(slot);
  const uint32_t* sm = reinterpret_cast<const uint32_t*>(slot + (size_t)R * nb * 16);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int NI = (nb + 31) / 32;
  int g = kMkConsumerWarps / max(R, 1);
  g = max(1, min(g, NI));
  const int groups = kMkConsumerWarps / g;
  if (w < groups * g) {
    const int slice = w % g;
    for (int rr = w / g; rr < R; rr += groups) {
      float acc = 0.f;
      for (int it = slice; it < NI; it += g) {
        const int b = lane + 32 * it;
        if (b < nb) {
          float scale, mn;
          unpack_sm(sm[(size_t)rr * nbp + b], scale, mn);
          const float A = q4_block_qx(qs[(size_t)rr * nb + b], S.xs, b);
          acc = fmaf(scale, A, fmaf(mn, S.xsum[b], acc));
        }
      }
      acc = warp_sum(acc);
      if (lane == 0) S.part[rr * g + slice] = acc;
    }
  }
  consumer_sync();
  for (int t = threadIdx.x; t < R; t += kMkConsumers) {
    float s = 0.f;
    for (int k = 0; k < g; ++k) s += S.part[t * g + k];
    rowsum[t] = flush_small(s);
  }
  consumer_sync();
}

// CTA-local lateral_inhibition_kwta on x[0..d): exact k-th largest by radix
// select, values below become -1e9 (the same mask in every CTA).
__device__ void mk_block_kwta(float* x, int d, int k, unsigned* hist) {
  const int tid = threadIdx.x;
  unsigned prefix = 0u, mask = 0u, kk = unsigned(k);
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kMkConsumers) hist[i] = 0u;
    consumer_sync();
    for (int i = tid; i < d; i += kMkConsumers) {
      const unsigned key = ord_key(x[i]);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xFFu], 1u);
    }
    consumer_sync();
    if (tid == 0) {
      unsigned acc = 0u;
      int b = 255;
      for (; b > 0; --b) {
        if (acc + hist[b] >= kk) break;
        acc += hist[b];
      }
      hist[256] = prefix | ((unsigned)b << shift);
      hist[257] = kk - acc;
    }
    consumer_sync();
    prefix = hist[256];
    kk = hist[257];
    mask |= 0xFFu << shift;
    consumer_sync();
  }
  const float thr = ord_val(prefix);
  for (int i = tid; i < d; i += kMkConsumers)
    if (x[i] < thr) x[i] = -1e9f;
  consumer_sync();
}

__device__ __forceinline__ void cta_units(const MkGemv& g, int& u0, int& u1) {
  u0 = blockIdx.x * g.upc;
  u1 = min(g.units, u0 + g.upc);
  if (u0 > u1) u0 = u1;
}

// Splits per KV head: at most one (head, split) unit per CTA.
__host__ __device__ inline int mk_split_cap(int nkv, int grid) {
  const int c = grid / nkv;
  return c < 1 ? 1 : (c > kAttnMaxSplits ? kAttnMaxSplits : c);
}

// Attention split owned by this CTA at context ctx (-1 if none).
__device__ __forceinline__ int attn_unit(int ctx, int nkv, int& nsplit, int& chunk) {
  attn_splits(ctx, nsplit, chunk, mk_split_cap(nkv, gridDim.x));
  const int units = nkv * nsplit;
  return (int)blockIdx.x < units ? (int)blockIdx.x : -1;
}

// ----------------------------------------------------------- producer
__device__ void mk_producer(const MegaArgs& A, const MkShared& S) {
  const StepParams& P = A.P;
  const MegaPlan& pl = A.plan;
  int item = 0;
  bool ok = true;
  auto issue = [&](const void* src0, uint32_t b0, const void* src1, uint32_t b1) {
    if (!ok) return;
    const int slot = item % pl.nslots;
    if (item >= pl.nslots && !mbar_wait(S.empty + slot, ((item / pl.nslots) - 1) & 1)) {
      flag_timeout(P.st, 11);
      *S.abort_flag = 1;
      ok = false;
      return;
    }
    if (*S.abort_flag || *S.cabort) {
      ok = false;
      return;
    }
    unsigned char* dst = S.slots + (size_t)slot * pl.slot_bytes;
    mbar_expect_tx(S.full + slot, b0 + b1);
    if (b0) bulk_g2s(dst, src0, b0, S.full + slot);
    if (b1) bulk_g2s(dst + b0, src1, b1, S.full + slot);
    ++item;
    *S.issued = item;
  };
  for (int step = 0; step < A.n_steps && ok; ++step) {
    for (int l = 0; l < P.n_layers && ok; ++l) {
      const LayerW& L = A.layers[l];
      const MkGemv* gs[4] = {&pl.q, &pl.o, &pl.g, &pl.d};
      const Q4View* ws[4] = {&L.qkv, &L.wo, &L.gate_up, &L.down};
      const int rpus[4] = {2, 1, 2, 1};
      for (int ph = 0; ph < 4 && ok; ++ph) {
        int u0, u1;
        cta_units(*gs[ph], u0, u1);
        const Q4View& W = *ws[ph];
        for (int a = u0; a < u1 && ok; a += gs[ph]->units_per_item) {
          const int ra = a * rpus[ph], nr = (min(u1, a + gs[ph]->units_per_item) - a) * rpus[ph];
          issue(W.qs + (size_t)ra * W.nb, uint32_t(nr) * W.nb * 16, W.sm + (size_t)ra * W.nbp,
                uint32_t(nr) * W.nbp * 4);
        }
      }
    }
    const int rbeg = blockIdx.x * pl.lm_rows_per_cta;
    const int rend = min(P.V, rbeg + pl.lm_rows_per_cta);
    for (int r = rbeg; r < rend && ok; r += pl.lm_stage_rows) {
      const int rows = min(pl.lm_stage_rows, rend - r);
      issue(P.lm_head + (size_t)r * P.d, uint32_t(rows) * P.d * 4, nullptr, 0u);
    }
  }
}

// ----------------------------------------------------------- consumers
// Every consumer thread waits (bounded) on the slot's full barrier; then all
// agree through a consumer barrier so that they return together on abort.
__device__ __forceinline__ const unsigned char* take(const MegaArgs& A, const MkShared& S, int item) {
  const int slot = item % A.plan.nslots;
  if (!mbar_wait(S.full + slot, (item / A.plan.nslots) & 1)) {
    flag_timeout(A.P.st, 12);
    *S.cabort = 1;
  }
  if (threadIdx.x == 0 && *S.abort_flag) *S.cabort = 1;
  consumer_sync();
  if (*S.cabort) return nullptr;
  return S.slots + (size_t)slot * A.plan.slot_bytes;
}
__device__ __forceinline__ void release(const MegaArgs& A, const MkShared& S, int item) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(S.empty + item % A.plan.nslots);
}
// Consumers agree on whether any of them failed (a bounded LL wait).
__device__ __forceinline__ bool agree(const MkShared& S, bool ok, DevState* st) {
  if (!ok) {
    flag_timeout(st, 13);
    *S.cabort = 1;
  }
  consumer_sync();
  return *S.cabort == 0;
}

__device__ void mk_consumer(const MegaArgs& A, const MkShared& S) {
  const StepParams& P = A.P;
  const MegaPlan& pl = A.plan;
  DevState* st = P.st;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int L = P.n_layers, d = P.d, hd = P.hd, half = hd >> 1;
  const int G = P.nh / P.nkv;
  __shared__ float red[32];
  __shared__ int redi[32];
  __shared__ unsigned hist[260];
  __shared__ unsigned long long wbest[32];
  __shared__ int is_last;
  __shared__ float mls[2 * kAttnMaxGroup];
  __shared__ float wsh[kAttnMaxGroup * kAttnMaxSplits];
  __shared__ float linv[kAttnMaxGroup];
  int item = 0;
  const unsigned pos0 = __ldcg(&st->pos);
  float* rowsum = S.part + 512;
  auto mark = [&](int step, int k) {
    if (A.phase_ns && blockIdx.x == 0 && tid == 0)
      A.phase_ns[(size_t)step * (5 * L + 1) + k] = global_ns();
  };
  auto tmark = [&](int step, int l, int ph, int k) {
    if (A.trace_ns && tid == 0)
      A.trace_ns[(((size_t)blockIdx.x * A.n_steps + step) * (5 * L + 1) + 5 * l + ph) * kMkTrace + k] = global_ns();
  };
  // one staged GEMV phase: items of this CTA's units, rows -> rowsum, epilogue per item
  auto gemv_phase = [&](const MkGemv& gp, const Q4View& W, int rpu, int step, int l, int ph,
                        auto&& epilogue) -> bool {
    int u0, u1;
    cta_units(gp, u0, u1);
    for (int a = u0; a < u1; a += gp.units_per_item) {
      const int b = min(u1, a + gp.units_per_item);
      const unsigned char* slot = take(A, S, item);
      if (!slot) return false;
      if (a == u0) tmark(step, l, ph, 3);
      mk_rows(S, slot, (b - a) * rpu, W.nb, W.nbp, rowsum);
      release(A, S, item++);
      epilogue(a, b);
      consumer_sync();  // rowsum is reused by the next item
    }
    return true;
  };

  // A CTA reads an exchanged vector only in phases where it has work whose
  // output other CTAs wait for: then every read of a buffer generation is
  // causally before the next generation's writes (no reader can be overtaken).
  int qa, qb, oa, ob, ga, gb, da, db;
  cta_units(pl.q, qa, qb);
  cta_units(pl.o, oa, ob);
  cta_units(pl.g, ga, gb);
  cta_units(pl.d, da, db);
  const bool has_q = qb > qa, has_o = ob > oa, has_g = gb > ga, has_d = db > da;
  for (int step = 0; step < A.n_steps; ++step) {
    const unsigned pos = pos0 + step;
    const int ctx = int(pos) + 1;
    int nsplit, chunk;
    const int au = attn_unit(ctx, P.nkv, nsplit, chunk);
    for (int l = 0; l < L; ++l) {
      const LayerW& Lw = A.layers[l];
      const unsigned e_qkv = mk_epoch(A.epoch0, L, step, l, 0), e_attn = e_qkv + 1, e_o = e_qkv + 2,
                     e_gu = e_qkv + 3, e_down = e_qkv + 4;
      // ================================================ QKV
      if (has_q || has_o || au >= 0) {
        tmark(step, l, 0, 0);
        // constant inputs first: norm weights, the RoPE row
        float wreg[kMkMaxNormVec];
#pragma unroll
        for (int k = 0; k < kMkMaxNormVec; ++k) {
          const int i = tid + k * kMkConsumers;
          wreg[k] = i < d ? Lw.attn_norm[i] : 0.f;
        }
        for (int i = tid; i < half; i += kMkConsumers) S.rope[i] = P.rope[(size_t)pos * half + i];
        float ss = 0.f;
        int bad = 0;
        bool ok = true;
        if (l == 0) {
          unsigned tok;
          if (step == 0) {
            tok = __ldcg(&st->token);
          } else {
            uint2 w = ld_ll(A.ll.tok);
            const unsigned e_prev = mk_epoch(A.epoch0, L, step - 1, L, 0);
            unsigned long long t0 = 0;
            while (w.y != e_prev) {
              const unsigned long long t = global_ns();
              if (!t0) t0 = t;
              else if (t - t0 > kWaitNs) {
                ok = false;
                break;
              }
              w = ld_ll(A.ll.tok);
            }
            fence_acq_rel_gpu();
            tok = w.x;
          }
          const float* src = P.embd + (size_t)(tok % (unsigned)P.V) * d;  // get_row_core: row token % V
          for (int i = tid; i < d; i += kMkConsumers) {
            const float v = __ldg(src + i);
            S.xraw[i] = v;
            ss = fmaf(v, v, ss);
            bad |= (v != v);
          }
        } else {
          ok = ll_read(A.ll.xb, d, mk_epoch(A.epoch0, L, step, l - 1, 4), S.xraw, ss, bad);
        }
        if (!agree(S, ok, st)) return;
        tmark(step, l, 0, 1);
        if (A.block_k > 0 && l > 0) {  // the previous block's K-WTA (block/forward.rs:145-149)
          mk_block_kwta(S.xraw, d, A.block_k, hist);
          ss = 0.f;
          for (int i = tid; i < d; i += kMkConsumers) ss = fmaf(S.xraw[i], S.xraw[i], ss);
        }
        for (int i = tid; i < d; i += kMkConsumers) S.xres[i] = S.xraw[i];
        const float tot = consumer_sum(ss, red);
        const int bad_in = consumer_any(bad, redi);
        const float inv = 1.0f / sqrtf(tot / (float)d + P.eps);
        int bad_out = 0;
        mk_stage_x(S, d, wreg, inv, true, bad_out);
        bad_out = consumer_any(bad_out, redi);  // also makes xs/xsum visible
        if (blockIdx.x == 0 && tid == 0) {
          if (bad_in) nan_flag(st, pos, l, kNanInput);
          if (bad_out) nan_flag(st, pos, l, kNanAttnNorm);
        }
        // this block's cached K/V rows for the attention split: every writer of
        // rows < pos finished before the x read above (acquire), so fetch now
        if (au >= 0 && tid == 0) {
          const int g = au % P.nkv, s = au / P.nkv, t0 = s * chunk;
          const int n = min(ctx, t0 + chunk) - t0;
          const int n_old = max(0, min(n, ctx - 1 - t0));
          const uint32_t bytes = uint32_t(n_old) * hd * 4;
          asm volatile("fence.proxy.async.global;" ::: "memory");
          *S.kv_armed = *S.kv_armed + 1;
          mbar_expect_tx(S.kv_bar, 2 * bytes);
          if (bytes) {
            bulk_g2s(S.kvbuf, Lw.kc + ((size_t)g * P.max_ctx + t0) * hd, bytes, S.kv_bar);
            bulk_g2s(S.kvbuf + (size_t)pl.attn_chunk_cap * hd, Lw.vc + ((size_t)g * P.max_ctx + t0) * hd, bytes,
                     S.kv_bar);
          }
        }
        tmark(step, l, 0, 2);
        const bool done = !has_q || gemv_phase(pl.q, Lw.qkv, 2, step, l, 0, [&](int a, int b) {
          for (int u = a + tid; u < b; u += kMkConsumers) {
            float y0 = rowsum[(u - a) * 2], y1 = rowsum[(u - a) * 2 + 1];
            if (Lw.qkv.bias) {
              y0 += Lw.qkv.bias[2 * u];
              y1 += Lw.qkv.bias[2 * u + 1];
            }
            const int head = u / half, i = u - head * half;
            const int c0 = P.rope_split ? i : 2 * i;
            const int c1 = P.rope_split ? i + half : 2 * i + 1;
            if (head < P.nh + P.nkv) {  // RoPE: v0*cos - v1*sin, v0*sin + v1*cos
              const float2 cs = S.rope[i];
              const float o0 = y0 * cs.x - y1 * cs.y;
              const float o1 = y0 * cs.y + y1 * cs.x;
              y0 = o0;
              y1 = o1;
            }
            uint2* dst = head < P.nh ? A.ll.q + head * hd
                                     : A.ll.kv + (head - P.nh) * hd;  // k heads then v heads
            st_ll(dst + c0, y0, e_qkv);
            st_ll(dst + c1, y1, e_qkv);
          }
        });
        if (!done) return;
        tmark(step, l, 0, 4);
        mark(step, 5 * l + 0);
      }
      // ================================================ ATTN
      if (au >= 0) {
        tmark(step, l, 1, 0);
        const int g = au % P.nkv, s = au / P.nkv, t0 = s * chunk;
        const int n = min(ctx, t0 + chunk) - t0;
        const int n_old = max(0, min(n, ctx - 1 - t0));
        const int cap = pl.attn_chunk_cap;
        float* Ks = S.kvbuf;
        float* Vs = S.kvbuf + (size_t)cap * hd;
        float* qs = S.xs;  // the group's q rows
        float dummy_ss = 0.f;
        int dummy_bad = 0;
        bool ok = ll_read(A.ll.q + (size_t)g * G * hd, G * hd, e_qkv, qs, dummy_ss, dummy_bad);
        if (ok && n > n_old) {  // this step's own row: LL, then into the cache for later steps
          const uint2* kn = A.ll.kv + (size_t)g * hd;
          const uint2* vn = A.ll.kv + (size_t)(P.nkv + g) * hd;
          ok = ll_read(kn, hd, e_qkv, Ks + (size_t)n_old * hd, dummy_ss, dummy_bad) &&
               ll_read(vn, hd, e_qkv, Vs + (size_t)n_old * hd, dummy_ss, dummy_bad);
          if (ok)
            for (int i = tid; i < hd; i += kMkConsumers) {
              Lw.kc[((size_t)g * P.max_ctx + pos) * hd + i] = Ks[(size_t)n_old * hd + i];
              Lw.vc[((size_t)g * P.max_ctx + pos) * hd + i] = Vs[(size_t)n_old * hd + i];
            }
        }
        tmark(step, l, 1, 1);
        // every consumer observes the copy's completion (parity of this use)
        const int use = *S.kv_waited;
        if (ok && !mbar_wait(S.kv_bar, use & 1)) ok = false;
        if (!agree(S, ok, st)) return;
        if (tid == 0) *S.kv_waited = use + 1;
        tmark(step, l, 1, 2);
        float* ps = S.ps;
        for (int idx = tid; idx < G * n; idx += kMkConsumers) {
          const int j = idx / n, t = idx - j * n;
          const float* qr = qs + j * hd;
          const float* kr = Ks + (size_t)t * hd;
          float a0 = 0.f, a1 = 0.f;
          int e0 = (t % hd) & ~1;
          for (int e = 0; e < hd; e += 2) {
            a0 = fmaf(qr[e0], kr[e0], a0);
            a1 = fmaf(qr[e0 + 1], kr[e0 + 1], a1);
            e0 += 2;
            if (e0 >= hd) e0 -= hd;
          }
          ps[j * chunk + t] = (a0 + a1) * P.attn_scale;
        }
        consumer_sync();
        for (int j = wid; j < G; j += kMkConsumerWarps) {
          float m = -INFINITY;
          for (int t = lane; t < n; t += kWarp) m = fmaxf(m, ps[j * chunk + t]);
          m = warp_max(m);
          float lsum = 0.f;
          for (int t = lane; t < n; t += kWarp) {
            const float ev = expf(ps[j * chunk + t] - m);
            ps[j * chunk + t] = ev;
            lsum += ev;
          }
          lsum = warp_sum(lsum);
          if (lane == 0) {
            mls[2 * j] = m;
            mls[2 * j + 1] = lsum;
          }
        }
        consumer_sync();
        const size_t pbase = ((size_t)g * kAttnMaxSplits + s) * G;
        for (int idx = tid; idx < G * hd; idx += kMkConsumers) {
          const int j = idx / hd, e = idx - j * hd;
          const float* pr = ps + j * chunk;
          float a0 = 0.f, a1 = 0.f;
          int t = 0;
          for (; t + 1 < n; t += 2) {
            a0 = fmaf(pr[t], Vs[(size_t)t * hd + e], a0);
            a1 = fmaf(pr[t + 1], Vs[(size_t)(t + 1) * hd + e], a1);
          }
          if (t < n) a0 = fmaf(pr[t], Vs[(size_t)t * hd + e], a0);
          P.part_o[(pbase + j) * hd + e] = a0 + a1;
        }
        if (tid < G) {
          P.part_ml[(pbase + tid) * 2] = mls[2 * tid];
          P.part_ml[(pbase + tid) * 2 + 1] = mls[2 * tid + 1];
        }
        __threadfence();  // partials and the new cache row before the arrival
        consumer_sync();
        tmark(step, l, 1, 3);
        if (tid == 0) is_last = (atomicAdd(P.attn_cnt + g, 1u) == (unsigned)nsplit - 1u);
        consumer_sync();
        if (is_last) {
          __threadfence();
          for (int idx = tid; idx < G * nsplit; idx += kMkConsumers) {
            const int j = idx / nsplit, r = idx - j * nsplit;
            wsh[idx] = __ldcg(P.part_ml + (((size_t)g * kAttnMaxSplits + r) * G + j) * 2);
          }
          consumer_sync();
          for (int j = wid; j < G; j += kMkConsumerWarps) {
            float M = -INFINITY;
            for (int r = lane; r < nsplit; r += kWarp) M = fmaxf(M, wsh[j * nsplit + r]);
            M = warp_max(M);
            float Ls = 0.f;
            for (int r = lane; r < nsplit; r += kWarp) {
              const float wgt = expf(wsh[j * nsplit + r] - M);
              wsh[j * nsplit + r] = wgt;
              Ls += __ldcg(P.part_ml + (((size_t)g * kAttnMaxSplits + r) * G + j) * 2 + 1) * wgt;
            }
            Ls = warp_sum(Ls);
            if (lane == 0) linv[j] = 1.0f / (Ls + 1e-12f);
          }
          consumer_sync();
          if (tid == 0) P.attn_cnt[g] = 0u;  // reset before the release below
          fence_acq_rel_gpu();
          for (int idx = tid; idx < G * hd; idx += kMkConsumers) {
            const int j = idx / hd, e = idx - j * hd;
            float O0 = 0.f, O1 = 0.f;
            int r = 0;
            for (; r + 1 < nsplit; r += 2) {
              O0 += __ldcg(P.part_o + (((size_t)g * kAttnMaxSplits + r) * G + j) * hd + e) * wsh[j * nsplit + r];
              O1 += __ldcg(P.part_o + (((size_t)g * kAttnMaxSplits + r + 1) * G + j) * hd + e) *
                    wsh[j * nsplit + r + 1];
            }
            if (r < nsplit)
              O0 += __ldcg(P.part_o + (((size_t)g * kAttnMaxSplits + r) * G + j) * hd + e) * wsh[j * nsplit + r];
            st_ll(A.ll.attn + ((size_t)g * G + j) * hd + e, (O0 + O1) * linv[j], e_attn);
          }
        }
        consumer_sync();
        tmark(step, l, 1, 4);
      }
      mark(step, 5 * l + 1);
      // ================================================ OPROJ
      if (has_o) {
        tmark(step, l, 2, 0);
        float ss = 0.f;
        int bad = 0;
        const bool ok = ll_read(A.ll.attn, Lw.wo.K, e_attn, S.xraw, ss, bad);
        if (!agree(S, ok, st)) return;
        tmark(step, l, 2, 1);
        int bo = 0;
        mk_stage_x(S, Lw.wo.K, nullptr, 1.0f, false, bo);
        consumer_sync();
        tmark(step, l, 2, 2);
        const bool done = gemv_phase(pl.o, Lw.wo, 1, step, l, 2, [&](int a, int b) {
          for (int r = a + tid; r < b; r += kMkConsumers) {
            float y = rowsum[r - a];
            if (Lw.wo.bias) y += Lw.wo.bias[r];
            st_ll(A.ll.xa + r, S.xres[r] + y, e_o);
          }
        });
        if (!done) return;
        tmark(step, l, 2, 4);
        mark(step, 5 * l + 2);
      }
      // ================================================ GATEUP
      if (has_g || has_d) {
        tmark(step, l, 3, 0);
        float wreg[kMkMaxNormVec];
#pragma unroll
        for (int k = 0; k < kMkMaxNormVec; ++k) {
          const int i = tid + k * kMkConsumers;
          wreg[k] = i < d ? Lw.ffn_norm[i] : 0.f;
        }
        float ss = 0.f;
        int bad = 0;
        const bool ok = ll_read(A.ll.xa, d, e_o, S.xraw, ss, bad);
        if (!agree(S, ok, st)) return;
        tmark(step, l, 3, 1);
        for (int i = tid; i < d; i += kMkConsumers) S.xres[i] = S.xraw[i];
        const float tot = consumer_sum(ss, red);
        const float inv = 1.0f / sqrtf(tot / (float)d + P.eps);
        int bo = 0;
        mk_stage_x(S, d, wreg, inv, true, bo);
        consumer_sync();
        tmark(step, l, 3, 2);
        const bool done = !has_g || gemv_phase(pl.g, Lw.gate_up, 2, step, l, 3, [&](int a, int b) {
          for (int u = a + tid; u < b; u += kMkConsumers) {
            float gv = rowsum[(u - a) * 2], uv = rowsum[(u - a) * 2 + 1];
            if (Lw.gate_up.bias) {
              gv += Lw.gate_up.bias[2 * u];
              uv += Lw.gate_up.bias[2 * u + 1];
            }
            if (uv != uv) nan_flag(st, pos, l, kNanUp);
            const float act = swiglu_balanced(gv, uv);
            if (act != act) nan_flag(st, pos, l, kNanFfnOut);
            st_ll(A.ll.act + u, act, e_gu);
          }
        });
        if (!done) return;
        tmark(step, l, 3, 4);
        mark(step, 5 * l + 3);
      }
      // ================================================ DOWN
      if (has_d) {
        tmark(step, l, 4, 0);
        float ss = 0.f;
        int bad = 0;
        const bool ok = ll_read(A.ll.act, P.ff, e_gu, S.xraw, ss, bad);
        if (!agree(S, ok, st)) return;
        tmark(step, l, 4, 1);
        float scale = 1.0f;
        if (P.use_genomic_norm) {  // block/forward.rs:115-123, h_scale = 1
          const float tot = consumer_sum(ss, red);
          const float rms = sqrtf(tot / (float)P.ff + P.eps);
          if (rms > 1.0f) scale = 1.0f / rms;
        }
        int bo = 0;
        if (scale != 1.0f)
          for (int i = tid; i < P.ff; i += kMkConsumers) S.xraw[i] = S.xraw[i] * scale;
        consumer_sync();
        mk_stage_x(S, P.ff, nullptr, 1.0f, false, bo);
        consumer_sync();
        tmark(step, l, 4, 2);
        const bool done = gemv_phase(pl.d, Lw.down, 1, step, l, 4, [&](int a, int b) {
          for (int r = a + tid; r < b; r += kMkConsumers) {
            float y = rowsum[r - a];
            if (Lw.down.bias) y += Lw.down.bias[r];
            if (y != y) nan_flag(st, pos, l, kNanProjFfn);
            const float xn = S.xres[r] + y;
            if (xn != xn) nan_flag(st, pos, l, kNanResidual);
            st_ll(A.ll.xb + r, xn, e_down);
          }
        });
        if (!done) return;
        tmark(step, l, 4, 4);
        mark(step, 5 * l + 4);
      }
    }
    // ================================================== LM
    {
      tmark(step, L, 0, 0);
      float wreg[kMkMaxNormVec];
#pragma unroll
      for (int k = 0; k < kMkMaxNormVec; ++k) {
        const int i = tid + k * kMkConsumers;
        wreg[k] = i < d ? P.out_norm[i] : 0.f;
      }
      float ss = 0.f;
      int bad = 0;
      const bool ok = ll_read(A.ll.xb, d, mk_epoch(A.epoch0, L, step, L - 1, 4), S.xraw, ss, bad);
      if (!agree(S, ok, st)) return;
      tmark(step, L, 0, 1);
      if (A.block_k > 0) {  // the last block's K-WTA
        mk_block_kwta(S.xraw, d, A.block_k, hist);
        ss = 0.f;
        for (int i = tid; i < d; i += kMkConsumers) ss = fmaf(S.xraw[i], S.xraw[i], ss);
      }
      const float tot = consumer_sum(ss, red);
      const float inv = 1.0f / sqrtf(tot / (float)d + P.eps);
      {
        int k = 0;
        for (int i = tid; i < d; i += kMkConsumers, ++k) S.xs[i] = (S.xraw[i] * inv) * wreg[k];  // plain layout
      }
      consumer_sync();
      tmark(step, L, 0, 2);
      const float4* x4 = reinterpret_cast<const float4*>(S.xs);
      const int K4 = d >> 2;
      unsigned long long best = 0ull;
      const int rbeg = blockIdx.x * pl.lm_rows_per_cta;
      const int rend = min(P.V, rbeg + pl.lm_rows_per_cta);
      for (int r = rbeg; r < rend; r += pl.lm_stage_rows) {
        const int rows = min(pl.lm_stage_rows, rend - r);
        const unsigned char* slot = take(A, S, item);
        if (!slot) return;
        if (r == rbeg) tmark(step, L, 0, 3);
        for (int rr = wid; rr < rows; rr += kMkConsumerWarps) {
          const float4* w4 = reinterpret_cast<const float4*>(slot) + (size_t)rr * K4;
          float a0 = 0.f, a1 = 0.f;
          for (int j = lane; j < K4; j += kWarp) {
            const float4 u = w4[j], xv = x4[j];
            a0 = fmaf(u.x, xv.x, a0);
            a1 = fmaf(u.y, xv.y, a1);
            a0 = fmaf(u.z, xv.z, a0);
            a1 = fmaf(u.w, xv.w, a1);
          }
          float sacc = warp_sum(a0 + a1);
          const int row = r + rr;
          if (P.lm_bias) sacc += P.lm_bias[row];
          if (lane == 0) P.logits[row] = sacc;
          const unsigned long long key = amax_key(sacc, (unsigned)row);
          best = key > best ? key : best;
        }
        release(A, S, item++);
      }
      best = warp_max_u64(best);
      if (lane == 0) wbest[wid] = best;
      consumer_sync();
      if (tid == 0) {
        unsigned long long b = 0;
        for (int i = 0; i < kMkConsumerWarps; ++i) b = wbest[i] > b ? wbest[i] : b;
        P.amax_part[blockIdx.x] = b;
        __threadfence();
        is_last = (atomicAdd(P.amax_cnt, 1u) == gridDim.x - 1u);
      }
      consumer_sync();
      if (is_last) {
        __threadfence();
        unsigned long long b = 0;
        for (int i = tid; i < (int)gridDim.x; i += kMkConsumers) {
          const unsigned long long v = __ldcg(P.amax_part + i);
          b = v > b ? v : b;
        }
        b = warp_max_u64(b);
        if (lane == 0) wbest[wid] = b;
        consumer_sync();
        if (tid == 0) {
          unsigned long long r = 0;
          for (int i = 0; i < kMkConsumerWarps; ++i) r = wbest[i] > r ? wbest[i] : r;
          const unsigned idx = amax_index(r);
          st->argmax = idx;
          st->token = idx;
          if (st->hist_len < P.hist_cap) P.tok_hist[st->hist_len] = idx;
          st->hist_len += 1u;
          st->pos = pos + 1u;
          *P.amax_cnt = 0u;
          fence_acq_rel_gpu();  // the state and the counter reset before the token word
          st_ll(A.ll.tok, __uint_as_float(idx), mk_epoch(A.epoch0, L, step, L, 0));
        }
      }
      consumer_sync();
      tmark(step, L, 0, 4);
      mark(step, 5 * L);
    }
  }
}

__global__ void __launch_bounds__(kMkThreads, 1) k_decode_mega(MegaArgs A) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const MegaPlan& pl = A.plan;
  const int hd = A.P.hd;
  MkShared S;
  S.full = reinterpret_cast<uint64_t*>(smem_raw);
  S.empty = S.full + kMkMaxSlots;
  S.kv_bar = S.empty + kMkMaxSlots;
  S.abort_flag = reinterpret_cast<volatile int*>(S.kv_bar + 1);
  S.issued = S.abort_flag + 1;
  S.cabort = S.abort_flag + 2;
  S.kv_armed = S.abort_flag + 3;
  S.kv_waited = S.abort_flag + 4;
  float* f = reinterpret_cast<float*>(smem_raw + kMkHeader);
  S.xs = f;
  f += pl.xs_floats;
  S.xraw = f;
  f += pl.xs_floats;
  S.xsum = f;
  f += pl.xs_floats / 32;
  S.xres = f;
  f += (A.P.d + 31) / 32 * 32;
  S.ps = f;
  f += pl.ps_floats;
  S.kvbuf = f;
  f += 2 * (size_t)pl.attn_chunk_cap * hd;
  S.part = f;
  f += kMkPartFloats;
  S.rope = reinterpret_cast<float2*>(f);
  f += hd;
  S.slots = reinterpret_cast<unsigned char*>(f);
  if (threadIdx.x == 0) {
    for (int i = 0; i < pl.nslots; ++i) {
      mbar_init(S.full + i, 1);
      mbar_init(S.empty + i, kMkConsumerWarps);
    }
    mbar_init(S.kv_bar, 1);
    *S.abort_flag = 0;
    *S.issued = 0;
    *S.cabort = 0;
    *S.kv_armed = 0;
    *S.kv_waited = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x >= kMkConsumers) {
    if (threadIdx.x == kMkConsumers) {
      mk_producer(A, S);
      // drain: every issued copy must land before the CTA may exit
      const int issued = *S.issued;
      for (int it = max(0, issued - pl.nslots); it < issued; ++it)
        mbar_wait(S.full + it % pl.nslots, (it / pl.nslots) & 1);
    }
    return;
  }
  mk_consumer(A, S);
  // an aborted block may leave its K/V copy in flight: it must land first
  if (threadIdx.x == 0 && *S.kv_armed > *S.kv_waited) mbar_wait(S.kv_bar, (*S.kv_waited) & 1);
}

}  // namespace gaje
