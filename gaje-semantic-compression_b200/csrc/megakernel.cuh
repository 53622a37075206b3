// megakernel.cuh -- persistent batch-1 decode: every phase of every block of
// GenomicLLM::forward_core (src/nn/llm/forward.rs:7-63), for n consecutive
// greedy steps, in one cooperative launch of one CTA per SM.
//
// Phases of a step, per block l:
//   QKV     attn_norm RMSNorm + attn_qkv GEMV + RoPE        -> q, new k/v
//   ATTN    split-K flash decode, one CTA per (KV head, split) -> split partials
//   OPROJ   combine of the split partials + attn_output GEMV + residual -> x_a
//   GATEUP  ffn_norm RMSNorm + ffn_gate_up GEMV + SwiGLU     -> act
//   DOWN    ffn_down GEMV + residual                         -> x_b (next block's x)
// then LM: output_norm + f32 lm_head GEMV + argmax            -> next token.
//
// No grid barriers.  Every vector a phase publishes goes to global memory as
// "LL" words: 8 bytes {float bits, epoch}, written and read as one 64-bit
// access, so a reader that sees the expected epoch also has the value.  A CTA
// starts a phase as soon as the words it needs carry the phase's epoch (a
// bounded spin); the all-to-all dependencies between phases order the reuse of
// each buffer.  The KV-cache rows (written by the attention CTA that owns the
// step's position, read a step or more later by TMA) and the argmax partials
// are ordered by fences.
//
// Warp roles: warps 0-14 compute ("consumers"); lane 0 of warp 15 is a
// producer that walks this CTA's static schedule of weight "items" (the rows
// of each GEMV phase, the lm_head row stages) and streams each item into a
// ring of shared-memory slots with 1-D TMA bulk copies (no multicast),
// full/empty mbarrier pairs per slot.  It runs up to a ring ahead of the
// consumers, so the next phases' weights are in flight while the consumers
// wait for activations.  The cached K/V rows of a CTA's attention split are
// fetched by the consumers themselves (TMA, at the start of the block's QKV
// phase).
//
// A phase on a CTA: warp 0 polls the publication flags of the CTAs that write
// the phase's input (the other warps wait on a named barrier), every consumer
// reads its share of the input words once and stages them in shared memory,
// one consumer barrier, the GEMV rows with no barrier, then warp 0 waits for
// the others' arrival (they do not wait) and raises this CTA's flag.  A warp
// passes the next phase's gate only after every warp finished this phase's
// rows, which is what lets the staged input be overwritten.
//
// RMSNorm is applied as x*w when staging and
// the 1/rms factor multiplies the finished row dot (the norm is linear in x),
// so staging is a single pass.  GEMV rows are taken by a warp per task: a
// row, or a row pair where the epilogue needs both rows (a RoPE pair, a
// gate/up pair; the pair shares its activation loads), lanes over the blocks,
// a shuffle reduction; a task's blocks are split over S warps with a
// shared-memory sum when a CTA has few long rows.  A lane's blocks form a
// serial dependency chain, so the mapping spends lanes before blocks.
//
// Q4_0 row dots (the AVX2 kernel's arithmetic, genomic.rs:267-336, factored):
// y = sum_b scale_b * A_b + min_b * X_b with A_b = sum_k q_k x_k and
// X_b = sum_k x_k.  q_k is obtained without shifting most nibbles: OR-ing the
// nibble found at bit position p of its word into the mantissa of 2^23 gives
// 2^23 + q*2^p exactly (p <= 16), and the activation is stored pre-scaled by
// 2^-p, so (f - 2^23) * x' = q * x exactly; the subtract and the FMA run as
// packed f32x2 instructions.
//
// Every wait is bounded (c_wait_ns); a wait that runs out sets DevState::err and
// the CTA's abort flag; the consumers leave together at their next barrier,
// the producer drains its in-flight copies (bounded) and exits.
#pragma once

#include "kernels.cuh"

namespace gaje {

constexpr int kMkThreads = 512;
constexpr int kMkConsumerWarps = 15;
constexpr int kMkConsumers = kMkConsumerWarps * 32;
constexpr int kMkMaxSlots = 8;
constexpr int kMkHeader = 1024;       // mbarriers + flags
constexpr int kMkPartFloats = 1024;   // split-K partials of a GEMV item
constexpr int kMkRound = 12;          // LL words per consumer thread per read round
constexpr int kMkMaxNormVec = 4;      // norm weights per thread (d <= 1920)
constexpr int kMkMinChunk = 64;       // positions per attention split (minimum)
constexpr int kMkCombine = 4;         // attention splits combined per read round
constexpr int kMkCombineElems = 2;    // attention outputs one consumer thread combines (n_head*head_dim <= 960)
// Trace points of a phase, per CTA: 0 entry, 1 input flags seen, 2 input
// staged (attention: cached K/V landed), 3 rows done (attention: scores
// done), 4 outputs published, 5 first weight slot ready.
constexpr int kMkTrace = 6;

// The vectors exchanged between phases, as {bits, epoch} words.
struct LLBufs {
  uint2* xa;     // [d] after the attention residual
  uint2* xb;     // [d] after the FFN residual (the next block's input)
  uint2* q;      // [nh*hd] rotated q
  uint2* kv;     // [2][nkv*hd] this step's k (rotated) and v rows
  uint2* apart;  // [nkv][max_splits][G][hd+2] attention split partials: o (unnormalised), m, l
  uint2* act;    // [ff] SwiGLU output
  uint2* tok;    // [1] the step's argmax (bits = token id)
  uint2* flags;  // [kFlCount][grid] per-CTA publication flags (epoch in .y)
};

// Publication flags: a CTA that wrote its share of a vector raises its flag
// (the vector's epoch) once all its consumer warps are past their stores; a
// reader polls the flags of the writer CTAs with one warp before it reads the
// vector's words once.  Polling a few flag words instead of the whole vector
// keeps the spinning CTAs off the L2 lines the data lives in.
enum MkFlag : int { kFlQkv = 0, kFlApart = 1, kFlXa = 2, kFlAct = 3, kFlXb = 4, kFlCount = 5 };

struct MkGemv {
  int units, upc, units_per_item;
};

struct MegaPlan {
  int nslots;
  unsigned slot_bytes;
  MkGemv q, o, g, d;
  int lm_rows_per_cta, lm_stage_rows;
  int xs_floats;    // activation buffers capacity (>= max K, multiple of 32)
  int ps_floats;    // attention scores capacity (G * chunk cap)
  int attn_chunk_cap;
  int qbuf_floats;  // G * hd
  int max_splits;   // attention splits per KV head (at most)
  int bias_floats;  // bias rows of one CTA in one GEMV phase (at most, multiple of 32)
  int layers_bytes; // the LayerW table copied to shared memory (multiple of 16)
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

__host__ __device__ inline int mk_round32(int n) { return (n + 31) / 32 * 32; }

__host__ __device__ inline size_t mega_smem_bytes(const MegaPlan& p, int d, int hd) {
  const size_t xs = p.xs_floats;
  return kMkHeader + size_t(p.layers_bytes) +
         4 * (xs + size_t(mk_round32(int(xs / 32))) + 2 * size_t(mk_round32(d)) + size_t(mk_round32(p.qbuf_floats)) + p.ps_floats +
              size_t(2) * p.attn_chunk_cap * hd + kMkPartFloats + 2 * hd + 2 * size_t(p.bias_floats)) +
         size_t(p.nslots) * p.slot_bytes;
}

// Splits per KV head: at most one (head, split) unit per CTA.
__host__ __device__ inline int mk_split_cap(int nkv, int grid) {
  const int c = grid / nkv;
  return c < 1 ? 1 : (c > kAttnMaxSplits ? kAttnMaxSplits : c);
}
__host__ __device__ inline void mk_attn_splits(int ctx, int max_splits, int& nsplit, int& chunk) {
  int n0 = (ctx + kMkMinChunk - 1) / kMkMinChunk;
  if (n0 > max_splits) n0 = max_splits;
  if (n0 < 1) n0 = 1;
  chunk = (ctx + n0 - 1) / n0;
  nsplit = (ctx + chunk - 1) / chunk;
}
__host__ __device__ inline int mk_chunk_cap(int max_ctx, int max_splits) {
  const int c = (max_ctx + max_splits - 1) / max_splits;
  return c > kMkMinChunk ? c : kMkMinChunk;
}

struct MkShared {
  uint64_t* full;
  uint64_t* empty;
  uint64_t* kv_bar;
  volatile int* abort_flag;  // raised by the producer
  volatile int* issued;      // items the producer has issued
  volatile int* cabort;      // consumers' abort decision (read after a consumer barrier)
  volatile int* kv_armed;    // uses of kv_bar armed so far (thread 0 of the consumers)
  volatile int* kv_waited;   // uses of kv_bar waited for
  float* xs;       // [xs_floats] staged GEMV input (x*w, pre-scaled, swizzled)
  float* xsum;     // [xs_floats/32] per-32-block sums of x*w
  float* xres[2];  // residual inputs: [0] of OPROJ (the block input), [1] of DOWN (x_a)
  float* qbuf;     // the attention group's q rows [G][hd]
  float* ps;       // attention scores [G][chunk cap]
  float* kvbuf;    // K rows [chunk cap][hd], then V rows
  float* part;     // split-K partials of a GEMV item
  float2* rope;    // the RoPE rows of the step's position, by step parity [2][hd/2]
  float* bias;     // [2][bias_floats] this CTA's bias rows of a GEMV phase, by phase parity
  const LayerW* layers;  // the LayerW table
  unsigned char* slots;
};

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kMkConsumers) : "memory"); }
__device__ __forceinline__ void bar_sync_n(int id) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(kMkConsumers) : "memory"); }
__device__ __forceinline__ void bar_arrive_n(int id) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(kMkConsumers) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ uint2 ld_ll(const uint2* p) {
  uint2 v;
  asm volatile("ld.relaxed.gpu.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_ll(uint2* p, float v, unsigned e) {
  asm volatile("st.relaxed.gpu.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(e) : "memory");
}

// Reads src[0..n) (LL words of epoch e) into raw[0..n) (shared memory):
// every consumer thread takes elements i = tid + k*480, R words in flight per
// round, and stores each once its round has arrived.  False if a word did not
// arrive in time.  Only loads, compares and stores are unrolled; whatever
// consumes the words runs afterwards, in a rolled loop over the same elements
// (keeping the persistent kernel's code small: it is re-fetched into the
// instruction cache in every phase).
template <int R>
__device__ __forceinline__ bool ll_gather(const uint2* src, int n, unsigned e, float* raw) {
  const int tid = threadIdx.x;
  for (int base = 0; base < n; base += R * kMkConsumers) {
    uint2 w[R];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const int i = base + tid + k * kMkConsumers;
      w[k] = i < n ? ld_ll(src + i) : make_uint2(0u, e);
    }
    unsigned long long t0 = 0;
    for (;;) {
      bool all = true;
#pragma unroll
      for (int k = 0; k < R; ++k) {
        if (w[k].y != e) {
          all = false;
          w[k] = ld_ll(src + base + tid + k * kMkConsumers);
        }
      }
      if (all) break;
      const unsigned long long t = global_ns();
      if (!t0) t0 = t;
      else if (t - t0 > c_wait_ns) return false;
    }
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const int i = base + tid + k * kMkConsumers;
      if (i < n) raw[i] = __uint_as_float(w[k].x);
    }
  }
  return true;
}

// Sum of v over the consumer threads, the same value (fixed order) in every
// thread; also the barrier that publishes what the consumers wrote before it.
// red: 16 floats, alternated between consecutive calls by the caller.
__device__ __forceinline__ float consumer_total(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[wid] = v;
  consumer_sync();
  float t = 0.f;
#pragma unroll
  for (int k = 0; k < kMkConsumerWarps; ++k) t += red[k];
  return t;
}

// End of a phase in which this CTA wrote words of a flagged vector: warp 0
// waits for the other consumer warps (named barrier 2; they do not wait) and
// raises the CTA's flag.
__device__ __forceinline__ void mk_publish(uint2* fl, unsigned e) {
  if (threadIdx.x < 32) {
    bar_sync_n(2);
    if (threadIdx.x == 0) st_ll(fl + blockIdx.x, 0.f, e);
  } else {
    bar_arrive_n(2);
  }
}
// Start of a phase reading a flagged vector written by CTAs [0, nw): warp 0
// polls their flags (bounded), the other warps wait for it (named barrier 3).
__device__ __forceinline__ void mk_gate(const uint2* fl, int nw, unsigned e, volatile int* cabort, DevState* st) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    bool ok = true;
    for (int base = 0; base < nw && ok; base += 32 * 8) {
      uint2 w[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = base + lane + 32 * k;
        w[k] = i < nw ? ld_ll(fl + i) : make_uint2(0u, e);
      }
      unsigned long long t0 = 0;
      for (;;) {
        bool all = true;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (w[k].y != e) {
            all = false;
            w[k] = ld_ll(fl + base + lane + 32 * k);
          }
        }
        if (all) break;
        const unsigned long long t = global_ns();
        if (!t0) t0 = t;
        else if (t - t0 > c_wait_ns) {
          ok = false;
          break;
        }
      }
    }
    if (!ok) {
      flag_timeout(st, 14);
      *cabort = 1;
    }
    __syncwarp();
    bar_arrive_n(3);
  } else {
    bar_sync_n(3);
  }
}

// 2^-p for the bit position p of element k (0..7) of a word: 0,4,8,12,16,8,12,16.
__device__ __forceinline__ float nib_prescale(int k) {
  const int p = k < 5 ? 4 * k : 4 * k - 12;
  return __int_as_float((127 - p) << 23);
}

// a[j] for a small register array and a run-time j < N.
template <int N>
__device__ __forceinline__ float pick(const float (&a)[N], int j) {
  float r = a[0];
#pragma unroll
  for (int k = 1; k < N; ++k)
    if (k == j) r = a[k];
  return r;
}

// One staged element: xs (swizzled, pre-scaled per nibble slot) and the
// block sums.  Called by whole warps (32 consecutive i).
__device__ __forceinline__ void mk_stage_elem(float* xs, float* xsum, int i, float xv) {
  xs[swz(i)] = xv * nib_prescale(i & 7);
  const float bs = warp_sum(xv);
  if ((threadIdx.x & 31) == 0) xsum[i >> 5] = bs;
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

// One 32-bit word (8 weights) of a block against its 8 pre-scaled
// activations, into two packed accumulators.
__device__ __forceinline__ void q4_word_qx(uint32_t a, const float4 xa, const float4 xb, unsigned long long& acc0,
                                           unsigned long long& acc1) {
  const uint32_t M = 0x4B000000u, t = a >> 12;
  const unsigned long long neg = pack2(-8388608.0f, -8388608.0f);
  const float f0 = __uint_as_float((a & 0xFu) | M), f1 = __uint_as_float((a & 0xF0u) | M);
  const float f2 = __uint_as_float((a & 0xF00u) | M), f3 = __uint_as_float((a & 0xF000u) | M);
  const float f4 = __uint_as_float((a & 0xF0000u) | M), f5 = __uint_as_float((t & 0xF00u) | M);
  const float f6 = __uint_as_float((t & 0xF000u) | M), f7 = __uint_as_float((t & 0xF0000u) | M);
  acc0 = ffma2(fadd2(pack2(f0, f1), neg), pack2(xa.x, xa.y), acc0);
  acc1 = ffma2(fadd2(pack2(f2, f3), neg), pack2(xa.z, xa.w), acc1);
  acc0 = ffma2(fadd2(pack2(f4, f5), neg), pack2(xb.x, xb.y), acc0);
  acc1 = ffma2(fadd2(pack2(f6, f7), neg), pack2(xb.z, xb.w), acc1);
}
__device__ __forceinline__ float hsum2(unsigned long long acc0, unsigned long long acc1) {
  float a0, a1, a2, a3;
  unpack2(acc0, a0, a1);
  unpack2(acc1, a2, a3);
  return (a0 + a1) + (a2 + a3);
}

// A = sum_k q_k x_k of one 32-weight block for two rows sharing the staged
// (swizzled, pre-scaled) activations of block b; the activations are loaded
// once, a word's worth at a time.
__device__ __forceinline__ void q4_pair_qx(const uint4 q0, const uint4 q1, bool has1, const float* xs, int b,
                                           float& A0, float& A1) {
  const float4* x4 = reinterpret_cast<const float4*>(xs + (b << 5));
  const int sw = b & 7;
  unsigned long long r00 = 0ull, r01 = 0ull, r10 = 0ull, r11 = 0ull;  // (+0.0f, +0.0f)
  const uint32_t w0[4] = {q0.x, q0.y, q0.z, q0.w};
  const uint32_t w1[4] = {q1.x, q1.y, q1.z, q1.w};
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const float4 xa = x4[(2 * w) ^ sw], xb = x4[(2 * w + 1) ^ sw];
    q4_word_qx(w0[w], xa, xb, r00, r01);
    if (has1) q4_word_qx(w1[w], xa, xb, r10, r11);
  }
  A0 = hsum2(r00, r01);
  A1 = hsum2(r10, r11);
}

// Work shape of one GEMV item of nr rows of nb blocks: tasks of rpt rows
// (rpt = 2 when the epilogue needs a row pair, or when single rows would not
// fit the lanes), 32 lanes per (task, slice) -- a lane's blocks are a serial
// chain, so the most lanes per task gives the shortest item -- and S slices
// of a task's blocks when lanes are left over and rows are long.
__device__ __forceinline__ void gemv_shape(int nr, int nb, bool pairs, int& rpt, int& S, int& tasks) {
  rpt = (pairs || nr * 32 > kMkConsumers) ? 2 : 1;
  tasks = (nr + rpt - 1) / rpt;
  S = 1;
  if (tasks * 64 <= kMkConsumers) S = max(1, min(kMkConsumers / (tasks * 32), nb / 48));
}

// CTA-local lateral_inhibition_kwta on x[0..d): exact k-th largest by radix
// select, values below become -1e9 (the same mask in every CTA).
__device__ __noinline__ void mk_block_kwta(float* x, int d, int k, unsigned* hist) {
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
// This CTA's bias rows of a GEMV phase into shared memory (zeros without a
// bias): the loads run while the phase waits for its input.
__device__ __forceinline__ float* mk_prefetch_bias(const MkShared& S, int bias_floats, const MkGemv& g,
                                                   const Q4View& W, int rpu, int par) {
  float* dst = S.bias + par * bias_floats;
  int u0, u1;
  cta_units(g, u0, u1);
  const int n = (u1 - u0) * rpu, r0 = u0 * rpu;
  const float* b = W.bias;
  for (int i = threadIdx.x; i < n; i += kMkConsumers) dst[i] = b ? __ldg(b + r0 + i) : 0.f;
  return dst;
}
// CTAs holding units of a GEMV phase: [0, writers).
__device__ __forceinline__ int mk_writers(const MkGemv& g) { return min((int)gridDim.x, (g.units + g.upc - 1) / g.upc); }

// Attention split owned by this CTA at context ctx (-1 if none).
__device__ __forceinline__ int attn_unit(int ctx, int nkv, int max_splits, int& nsplit, int& chunk) {
  mk_attn_splits(ctx, max_splits, nsplit, chunk);
  const int units = nkv * nsplit;
  return (int)blockIdx.x < units ? (int)blockIdx.x : -1;
}

// ----------------------------------------------------------- producer
// Walks the item sequence a step consumes -- per block, the units of each
// GEMV phase (QKV, O-proj, gate/up, down) in items of units_per_item, then the
// lm_head rows in stages -- and streams every item into the next ring slot.
__device__ void mk_producer(const MegaArgs& A, const MkShared& S) {
  const StepParams& P = A.P;
  const MegaPlan& pl = A.plan;
  const int L = P.n_layers;
  const int rbeg = blockIdx.x * pl.lm_rows_per_cta, rend = min(P.V, rbeg + pl.lm_rows_per_cta);
  int item = 0;
  for (int step = 0; step < A.n_steps; ++step) {
    int l = 0, ph = 0, a = -1, r = rbeg;
    for (;;) {
      const void* src0;
      const void* src1 = nullptr;
      uint32_t b0, b1 = 0u;
      if (l < L) {
        const MkGemv& g = ph == 0 ? pl.q : ph == 1 ? pl.o : ph == 2 ? pl.g : pl.d;
        int u0, u1;
        cta_units(g, u0, u1);
        if (a < 0) a = u0;
        if (a >= u1) {
          a = -1;
          if (++ph == 4) {
            ph = 0;
            ++l;
          }
          continue;
        }
        const LayerW& Lw = A.layers[l];
        const Q4View& W = ph == 0 ? Lw.qkv : ph == 1 ? Lw.wo : ph == 2 ? Lw.gate_up : Lw.down;
        const int rpu = (ph == 0 || ph == 2) ? 2 : 1;
        const int ra = a * rpu, nr = (min(u1, a + g.units_per_item) - a) * rpu;
        src0 = W.qs + (size_t)ra * W.nb;
        b0 = uint32_t(nr) * W.nb * 16;
        src1 = W.sm + (size_t)ra * W.nbp;
        b1 = uint32_t(nr) * W.nbp * 4;
        a += g.units_per_item;
      } else {
        if (r >= rend) break;
        const int rows = min(pl.lm_stage_rows, rend - r);
        src0 = P.lm_head + (size_t)r * P.d;
        b0 = uint32_t(rows) * P.d * 4;
        r += pl.lm_stage_rows;
      }
      const int slot = item % pl.nslots;
      if (item >= pl.nslots && !mbar_wait(S.empty + slot, ((item / pl.nslots) - 1) & 1)) {
        flag_timeout(P.st, 11);
        *S.abort_flag = 1;
        return;
      }
      if (*S.abort_flag || *S.cabort) return;
      unsigned char* dst = S.slots + (size_t)slot * pl.slot_bytes;
      mbar_expect_tx(S.full + slot, b0 + b1);
      bulk_g2s(dst, src0, b0, S.full + slot);
      if (b1) bulk_g2s(dst + b0, src1, b1, S.full + slot);
      ++item;
      *S.issued = item;
    }
  }
}

// ----------------------------------------------------------- consumers
// Every consumer thread waits (bounded) for the item's slot; a wait that runs
// out raises the abort flag, which the consumers act on at their next barrier.
__device__ __forceinline__ const unsigned char* wait_slot(const MegaArgs& A, const MkShared& S, int item) {
  const int slot = item % A.plan.nslots;
  if (!*S.cabort && !*S.abort_flag && !mbar_wait(S.full + slot, (item / A.plan.nslots) & 1)) {
    flag_timeout(A.P.st, 12);
    *S.cabort = 1;
  }
  if (*S.abort_flag) *S.cabort = 1;
  return S.slots + (size_t)slot * A.plan.slot_bytes;
}
__device__ __forceinline__ void release(const MegaArgs& A, const MkShared& S, int item) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(S.empty + item % A.plan.nslots);
}

// One GEMV phase of this CTA: its units in staged items, each item's rows
// dotted against xs/xsum, a warp per (task, slice); epi(a, r, y0, y1, has1)
// gets the raw dots of the item's local rows r and r+1 (r+1 when has1) of the
// item starting at unit a (its first row is a*rpu).  The epilogue has one
// call site (the kernel's code size matters).
template <class Epi>
__device__ __forceinline__ void mk_gemv(const MegaArgs& A, const MkShared& S, const MkGemv& gp, const Q4View& W,
                                        int rpu, const float* xs, const float* xsum, int& item,
                                        unsigned long long* first_ready, Epi&& epi) {
  const int tid = threadIdx.x, lane = tid & 31, gid = tid >> 5;
  int u0, u1;
  cta_units(gp, u0, u1);
  const int nb = W.nb, nbp = W.nbp;
  for (int a = u0; a < u1; a += gp.units_per_item) {
    const int nr = (min(u1, a + gp.units_per_item) - a) * rpu;
    const unsigned char* slot = wait_slot(A, S, item);
    if (first_ready && a == u0 && tid == 0) *first_ready = global_ns();
    const uint4* qs = reinterpret_cast<const uint4*>(slot);
    const uint32_t* sm = reinterpret_cast<const uint32_t*>(slot + (size_t)nr * nb * 16);
    int rpt, Sl, tasks;
    gemv_shape(nr, nb, rpu == 2, rpt, Sl, tasks);
    const int nts = tasks * Sl;
    // with slices every warp runs one round (a barrier joins the slices)
    const int iters = Sl > 1 ? 1 : (gid < nts ? (nts - gid + kMkConsumerWarps - 1) / kMkConsumerWarps : 0);
    for (int it = 0; it < iters; ++it) {
      const int ts = gid + it * kMkConsumerWarps;
      int p = ts / Sl;
      const int sl = ts - p * Sl;
      float acc0 = 0.f, acc1 = 0.f;
      if (ts < nts) {
        const int r0 = rpt * p;
        const bool h1 = rpt == 2 && r0 + 1 < nr;
        for (int b = sl * 32 + lane; b < nb; b += Sl * 32) {
          const uint4 q0 = qs[(size_t)r0 * nb + b];
          const uint4 q1 = h1 ? qs[(size_t)(r0 + 1) * nb + b] : make_uint4(0u, 0u, 0u, 0u);
          const uint32_t sm0 = sm[(size_t)r0 * nbp + b], sm1 = h1 ? sm[(size_t)(r0 + 1) * nbp + b] : 0u;
          const float xb = xsum[b];
          float A0, A1, sc, mn;
          q4_pair_qx(q0, q1, h1, xs, b, A0, A1);
          unpack_sm(sm0, sc, mn);
          acc0 = fmaf(sc, A0, fmaf(mn, xb, acc0));
          unpack_sm(sm1, sc, mn);
          acc1 = fmaf(sc, A1, fmaf(mn, xb, acc1));
        }
        acc0 = warp_sum(acc0);
        acc1 = warp_sum(acc1);
      }
      bool fire = ts < nts && lane == 0;
      if (Sl > 1) {  // uniform over the CTA: the slices' partials, summed in slice order
        if (fire) {
          S.part[2 * ts] = acc0;
          S.part[2 * ts + 1] = acc1;
        }
        consumer_sync();
        p = gid;
        fire = gid < tasks && lane == 0;
        if (fire) {
          acc0 = 0.f;
          acc1 = 0.f;
          for (int s = 0; s < Sl; ++s) {
            acc0 += S.part[2 * (p * Sl + s)];
            acc1 += S.part[2 * (p * Sl + s) + 1];
          }
        }
      }
      if (fire) epi(a, rpt * p, acc0, acc1, rpt == 2 && rpt * p + 1 < nr);
    }
    release(A, S, item++);
    if (Sl > 1) consumer_sync();  // the partials buffer is reused by the next item
  }
}

// Phases of a block, in order, and the step's lm_head phase.
enum MkPhase : int { kPhQkv = 0, kPhAttn = 1, kPhOproj = 2, kPhGateup = 3, kPhDown = 4, kPhLm = 5 };

__device__ void mk_consumer(const MegaArgs& A, const MkShared& S) {
  const StepParams& P = A.P;
  const MegaPlan& pl = A.plan;
  DevState* st = P.st;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int L = P.n_layers, d = P.d, hd = P.hd, half = hd >> 1;
  const int G = P.nh / P.nkv, qd = P.nh * P.hd;
  const int Smax = pl.max_splits, cap = pl.attn_chunk_cap;
  __shared__ float red[2][16];
  __shared__ unsigned hist[260];
  __shared__ unsigned long long wbest[32];
  __shared__ int is_last;
  __shared__ float mls[2 * kAttnMaxGroup];
  int item = 0, ph_count = 0;
  const unsigned pos0 = __ldcg(&st->pos);
  auto tmark = [&](int step, int pi, int k) {
    if (A.trace_ns && tid == 0)
      A.trace_ns[(((size_t)blockIdx.x * A.n_steps + step) * (5 * L + 1) + pi) * kMkTrace + k] = global_ns();
  };
  // A CTA reads an exchanged vector only in phases where it has work whose
  // output other CTAs wait for: then every read of a buffer generation is
  // causally before the next generation's writes (no reader can be overtaken).
  auto has = [&](const MkGemv& g) { return (int)blockIdx.x * g.upc < g.units; };
  const bool has_q = has(pl.q), has_o = has(pl.o), has_g = has(pl.g), has_d = has(pl.d);
  for (int step = 0; step < A.n_steps; ++step) {
    const unsigned pos = pos0 + step;
    const int ctx = int(pos) + 1;
    int nsplit, chunk;
    const int au = attn_unit(ctx, P.nkv, Smax, nsplit, chunk);
    float2* rope = S.rope + (step & 1) * half;  // by step parity: no reader of the previous row is left
    // phase index pi = 5l + ph over the blocks, then pi = 5L: the lm_head
    for (int pi = 0; pi <= 5 * L; ++pi) {
      const int l = pi < 5 * L ? pi / 5 : L - 1;
      const int ph = pi < 5 * L ? pi - 5 * l : int(kPhLm);
      const LayerW& Lw = S.layers[l];
      const unsigned e_qkv = mk_epoch(A.epoch0, L, step, l, 0), e_attn = e_qkv + 1;
      if (ph == kPhAttn) {
        // ============================================== ATTN
        if (au >= 0) {
          tmark(step, pi, 0);
          const int g = au % P.nkv, s = au / P.nkv, t0 = s * chunk;
          const int n = min(ctx, t0 + chunk) - t0;
          const int n_old = max(0, min(n, ctx - 1 - t0));
          float* Ks = S.kvbuf;
          float* Vs = S.kvbuf + (size_t)cap * hd;
          mk_gate(A.ll.flags + kFlQkv * gridDim.x, mk_writers(pl.q), e_qkv, S.cabort, st);
          tmark(step, pi, 1);
          bool ok = ll_gather<2>(A.ll.q + (size_t)g * G * hd, G * hd, e_qkv, S.qbuf);
          if (n > n_old)  // this step's own row: LL, then into the cache for later steps
            ok = ok && ll_gather<2>(A.ll.kv + (size_t)g * hd, hd, e_qkv, Ks + (size_t)n_old * hd) &&
                 ll_gather<2>(A.ll.kv + (size_t)(P.nkv + g) * hd, hd, e_qkv, Vs + (size_t)n_old * hd);
          const bool wrote_row = ok && n > n_old && tid < hd;
          if (wrote_row) {
            Lw.kc[((size_t)g * P.max_ctx + pos) * hd + tid] = Ks[(size_t)n_old * hd + tid];
            Lw.vc[((size_t)g * P.max_ctx + pos) * hd + tid] = Vs[(size_t)n_old * hd + tid];
          }
          // every consumer observes the copy's completion (parity of this use)
          const int use = *S.kv_waited;
          if (ok && !*S.cabort && !mbar_wait(S.kv_bar, use & 1)) ok = false;
          if (!ok) {
            flag_timeout(st, 13);
            *S.cabort = 1;
          }
          consumer_sync();
          if (*S.cabort) return;
          if (tid == 0) *S.kv_waited = use + 1;
          tmark(step, pi, 2);
          // scores: lane = position, warps over (32-position block, head subset)
          {
            const int npb = (n + 31) >> 5;
            const int nhs = max(1, min(G, kMkConsumerWarps / npb));
            const int H4 = hd >> 2;
            for (int task = wid; task < npb * nhs; task += kMkConsumerWarps) {
              const int pb = task % npb, hs = task / npb;
              const int t = pb * 32 + lane;
              if (t < n) {
                const float4* kr = reinterpret_cast<const float4*>(Ks + (size_t)t * hd);
                for (int j = hs; j < G; j += nhs) {
                  const float4* qr = reinterpret_cast<const float4*>(S.qbuf + j * hd);
                  float a0 = 0.f, a1 = 0.f;
                  int c = lane % H4;  // rotated start: conflict-free rows
                  for (int k = 0; k < H4; ++k) {
                    const float4 kk = kr[c], qq = qr[c];
                    a0 = fmaf(qq.x, kk.x, a0);
                    a1 = fmaf(qq.y, kk.y, a1);
                    a0 = fmaf(qq.z, kk.z, a0);
                    a1 = fmaf(qq.w, kk.w, a1);
                    c = c + 1 == H4 ? 0 : c + 1;
                  }
                  S.ps[j * cap + t] = (a0 + a1) * P.attn_scale;
                }
              }
            }
          }
          if (wrote_row) __threadfence();  // the new cache row before this split's partials
          consumer_sync();
          tmark(step, pi, 3);
          for (int j = wid; j < G; j += kMkConsumerWarps) {
            float* pr = S.ps + j * cap;
            float m = -INFINITY;
            for (int t = lane; t < n; t += kWarp) m = fmaxf(m, pr[t]);
            m = warp_max(m);
            float lsum = 0.f;
            for (int t = lane; t < n; t += kWarp) {
              const float ev = expf(pr[t] - m);
              pr[t] = ev;
              lsum += ev;
            }
            lsum = warp_sum(lsum);
            if (lane == 0) {
              mls[2 * j] = m;
              mls[2 * j + 1] = lsum;
            }
          }
          consumer_sync();
          uint2* part = A.ll.apart + ((size_t)g * Smax + s) * G * (hd + 2);
          for (int idx = tid; idx < G * hd; idx += kMkConsumers) {
            const int j = idx / hd, e = idx - j * hd;
            const float* pr = S.ps + j * cap;
            float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
            int t = 0;
            for (; t + 3 < n; t += 4) {
              o0 = fmaf(pr[t], Vs[(size_t)t * hd + e], o0);
              o1 = fmaf(pr[t + 1], Vs[(size_t)(t + 1) * hd + e], o1);
              o2 = fmaf(pr[t + 2], Vs[(size_t)(t + 2) * hd + e], o2);
              o3 = fmaf(pr[t + 3], Vs[(size_t)(t + 3) * hd + e], o3);
            }
            for (; t < n; ++t) o0 = fmaf(pr[t], Vs[(size_t)t * hd + e], o0);
            uint2* pj = part + (size_t)j * (hd + 2);
            st_ll(pj + e, (o0 + o1) + (o2 + o3), e_attn);
            if (e == 0) {
              st_ll(pj + hd, mls[2 * j], e_attn);
              st_ll(pj + hd + 1, mls[2 * j + 1], e_attn);
            }
          }
          mk_publish(A.ll.flags + kFlApart * gridDim.x, e_attn);
          tmark(step, pi, 4);
        }
        if (A.phase_ns && blockIdx.x == 0 && tid == 0) A.phase_ns[(size_t)step * (5 * L + 1) + pi] = global_ns();
        continue;
      }
      // ================================================ GEMV phases and LM
      // QKV     attn_norm(x) -> qkv rows + RoPE -> q, k, v      (in: x_b of block l-1)
      // OPROJ   attention combine -> attn_output rows + x      (in: split partials)
      // GATEUP  ffn_norm(x_a) -> gate/up rows + SwiGLU -> act   (in: x_a)
      // DOWN    act -> ffn_down rows + x_a -> x_b               (in: act)
      // LM      output_norm(x_b) -> lm_head rows -> argmax      (in: x_b of block L-1)
      const bool stage_here = ph == kPhQkv ? (has_q || has_o || au >= 0)
                              : ph == kPhOproj ? has_o : ph == kPhGateup ? (has_g || has_d)
                              : ph == kPhDown ? has_d : true;
      if (!stage_here) continue;
      tmark(step, pi, 0);
      const MkGemv& gp = ph == kPhQkv ? pl.q : ph == kPhOproj ? pl.o : ph == kPhGateup ? pl.g : pl.d;
      const Q4View& W = ph == kPhQkv ? Lw.qkv : ph == kPhOproj ? Lw.wo : ph == kPhGateup ? Lw.gate_up : Lw.down;
      const int rpu = (ph == kPhQkv || ph == kPhGateup) ? 2 : 1;
      const float* norm = ph == kPhQkv ? Lw.attn_norm : ph == kPhGateup ? Lw.ffn_norm : ph == kPhLm ? P.out_norm : nullptr;
      // raw input: the residual copies for QKV / GATEUP, xres[0] for LM (free
      // again: last read by the last block's O-proj), xs itself for DOWN
      float* raw = ph == kPhGateup ? S.xres[1] : ph == kPhDown ? S.xs : S.xres[0];
      const unsigned e_out = e_qkv + unsigned(ph);
      const int K = ph == kPhDown ? P.ff : ph == kPhOproj ? qd : d;
      float wreg[kMkMaxNormVec];
#pragma unroll
      for (int k = 0; k < kMkMaxNormVec; ++k) {
        const int i = tid + k * kMkConsumers;
        wreg[k] = norm && i < d ? norm[i] : 1.f;
      }
      if (ph == kPhQkv && l == 0)
        for (int i = tid; i < half; i += kMkConsumers) rope[i] = P.rope[(size_t)pos * half + i];
      const float* bsm = ph == kPhLm ? nullptr : mk_prefetch_bias(S, pl.bias_floats, gp, W, rpu, ph_count & 1);
      float* xs = S.xs;
      float* xsum = S.xsum;
      float ss = 0.f;
      bool ok = true;
      if (ph == kPhOproj) {
        mk_gate(A.ll.flags + kFlApart * gridDim.x, P.nkv * nsplit, e_attn, S.cabort, st);
        tmark(step, pi, 1);
        // combine of the split partials (the softmax of attention.rs:88-127
        // across splits): weights exp(m_s - M), out = O / (L + 1e-12).  Per
        // round of kMkCombine splits every word is requested at once: the
        // (m, l) pairs by one thread each into shared memory, the o words of
        // this thread's elements (at most kMkCombineElems; plan_mega rejects
        // larger n_head * head_dim) into registers.
        constexpr int kE = kMkCombineElems;
        float M[kE], O[kE], Ls[kE];
        const uint2* ob[kE];
#pragma unroll
        for (int j = 0; j < kE; ++j) {
          M[j] = -INFINITY;
          O[j] = 0.f;
          Ls[j] = 0.f;
          const int i = min(tid + j * kMkConsumers, qd - 1);
          const int h = i / hd, e = i - h * hd;
          const int g = h / G, jh = h - g * G;
          ob[j] = A.ll.apart + ((size_t)g * Smax * G + jh) * (hd + 2) + e;
        }
        const uint2* pml = nullptr;
        if (tid < P.nh * kMkCombine) {
          const int h = tid / kMkCombine, g = h / G, jh = h - g * G;
          pml = A.ll.apart + ((size_t)g * Smax * G + jh) * (hd + 2) + hd + (size_t)(tid % kMkCombine) * G * (hd + 2);
        }
        const size_t sstride = (size_t)G * (hd + 2);
        for (int s0 = 0; s0 < nsplit; s0 += kMkCombine) {
          const int ns = min(kMkCombine, nsplit - s0);
          float* mlp = S.part;  // [nh][kMkCombine][2]
          const bool mine = pml && tid % kMkCombine < ns;
          const uint2* pm = pml + (size_t)s0 * sstride;
          uint2 wm = mine ? ld_ll(pm) : make_uint2(0u, e_attn), wl = mine ? ld_ll(pm + 1) : make_uint2(0u, e_attn);
          uint2 wo[kE][kMkCombine];
#pragma unroll
          for (int j = 0; j < kE; ++j) {
            const bool live = tid + j * kMkConsumers < qd;
#pragma unroll
            for (int k = 0; k < kMkCombine; ++k)
              wo[j][k] = (live && k < ns) ? ld_ll(ob[j] + (size_t)(s0 + k) * sstride) : make_uint2(0u, e_attn);
          }
          unsigned long long tw = 0;
          for (;;) {
            bool all = true;
            if (wm.y != e_attn) {
              all = false;
              wm = ld_ll(pm);
            }
            if (wl.y != e_attn) {
              all = false;
              wl = ld_ll(pm + 1);
            }
#pragma unroll
            for (int j = 0; j < kE; ++j)
#pragma unroll
              for (int k = 0; k < kMkCombine; ++k)
                if (wo[j][k].y != e_attn) {
                  all = false;
                  wo[j][k] = ld_ll(ob[j] + (size_t)(s0 + k) * sstride);
                }
            if (all) break;
            const unsigned long long t = global_ns();
            if (!tw) tw = t;
            else if (t - tw > c_wait_ns) {
              ok = false;
              break;
            }
          }
          if (mine) {
            mlp[tid * 2] = __uint_as_float(wm.x);
            mlp[tid * 2 + 1] = __uint_as_float(wl.x);
          }
          consumer_sync();
#pragma unroll
          for (int j = 0; j < kE; ++j) {
            const int i = tid + j * kMkConsumers;
            if (i >= qd) break;
            const float* ml = mlp + (i / hd) * kMkCombine * 2;
            float Mn = M[j];
            for (int k = 0; k < ns; ++k) Mn = fmaxf(Mn, ml[2 * k]);
            const float r = expf(M[j] - Mn);  // 0 on the first round (M = -inf)
            O[j] *= r;
            Ls[j] *= r;
#pragma unroll
            for (int k = 0; k < kMkCombine; ++k) {
              if (k < ns) {
                const float w = expf(ml[2 * k] - Mn);
                O[j] = fmaf(__uint_as_float(wo[j][k].x), w, O[j]);
                Ls[j] = fmaf(ml[2 * k + 1], w, Ls[j]);
              }
            }
            M[j] = Mn;
          }
          if (s0 + kMkCombine < nsplit) consumer_sync();  // the (m, l) buffer is refilled
        }
#pragma unroll
        for (int j = 0; j < kE; ++j) {
          const int i = tid + j * kMkConsumers;
          if (i < qd) mk_stage_elem(xs, xsum, i, O[j] * (1.0f / (Ls[j] + 1e-12f)));
        }
      } else {
        // the input vector into raw: the step's embedding row (QKV of block
        // 0) or the flagged LL words of the previous phase
        if (ph == kPhQkv && l == 0) {
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
              else if (t - t0 > c_wait_ns) {
                ok = false;
                break;
              }
              w = ld_ll(A.ll.tok);
            }
            tok = w.x;
          }
          tmark(step, pi, 1);
          const float* src = P.embd + (size_t)(tok % (unsigned)P.V) * d;  // get_row_core: row token % V
          for (int i = tid; i < d; i += kMkConsumers) raw[i] = __ldg(src + i);
        } else {
          const int fl = ph == kPhGateup ? kFlXa : ph == kPhDown ? kFlAct : kFlXb;
          const int nw = mk_writers(ph == kPhGateup ? pl.o : ph == kPhDown ? pl.g : pl.d);
          const unsigned e_in = ph == kPhLm ? mk_epoch(A.epoch0, L, step, L - 1, 4) : e_out - 1;
          const uint2* src = ph == kPhGateup ? A.ll.xa : ph == kPhDown ? A.ll.act : A.ll.xb;
          mk_gate(A.ll.flags + fl * gridDim.x, nw, e_in, S.cabort, st);
          tmark(step, pi, 1);
          ok = ll_gather<kMkRound>(src, K, e_in, raw);
          // the previous block's K-WTA (block/forward.rs:145-149; the last
          // block's before the output norm)
          if ((ph == kPhQkv || ph == kPhLm) && A.block_k > 0) {
            if (!ok) *S.cabort = 1;
            consumer_sync();
            if (*S.cabort) return;
            mk_block_kwta(raw, d, A.block_k, hist);
          }
        }
        // one staging pass: x*w (pre-scaled, swizzled, with block sums) for
        // the Q4 GEMVs; plain x*w for the f32 lm_head
        const bool plain = ph == kPhLm;
        for (int j = 0, i = tid; i < K; i += kMkConsumers, ++j) {
          const float v = raw[i];
          ss = fmaf(v, v, ss);
          const float xv = v * pick(wreg, j);
          if (plain) {
            xs[i] = xv;
          } else {
            __syncwarp();  // DOWN stages in place: the warp's block is read before it is permuted
            mk_stage_elem(xs, xsum, i, xv);
          }
        }
      }
      float tot;
      if (!ok) {
        flag_timeout(st, 13);
        *S.cabort = 1;
      }
      tot = consumer_total(ss, red[ph_count & 1]);
      ++ph_count;
      if (*S.cabort) return;
      tmark(step, pi, 2);
      // the norm's 1/rms (QKV, GATEUP, LM) or the genomic scale (DOWN) of the row dots
      float scale = 1.0f;
      if (norm) scale = 1.0f / sqrtf(tot / (float)d + P.eps);
      if (ph == kPhDown && P.use_genomic_norm) {  // block/forward.rs:115-123, h_scale = 1
        const float rms = sqrtf(tot / (float)P.ff + P.eps);
        if (rms > 1.0f) scale = 1.0f / rms;
      }
      if (ph == kPhLm) {
        // ============================================ lm_head + argmax
        const float4* x4 = reinterpret_cast<const float4*>(xs);
        const int K4 = d >> 2;
        unsigned long long best = 0ull;
        const int rbeg = blockIdx.x * pl.lm_rows_per_cta;
        const int nrows = max(0, min(P.V, rbeg + pl.lm_rows_per_cta) - rbeg);
        const int nitems = (nrows + pl.lm_stage_rows - 1) / pl.lm_stage_rows;
        // warp w takes rows w, w+15, ...; it waits for (and releases) every
        // stage in order, also the ones holding none of its rows
        int cur = -1;
        const unsigned char* slot = nullptr;
        for (int k = wid; k < nrows; k += kMkConsumerWarps) {
          const int it = k / pl.lm_stage_rows;
          while (cur < it) {
            if (cur >= 0) release(A, S, item + cur);
            ++cur;
            slot = wait_slot(A, S, item + cur);
          }
          if (k == 0) tmark(step, pi, 5);
          const float4* w4 = reinterpret_cast<const float4*>(slot) + (size_t)(k - it * pl.lm_stage_rows) * K4;
          float a0 = 0.f, a1 = 0.f;
          for (int j = lane; j < K4; j += kWarp) {
            const float4 u = w4[j], xv = x4[j];
            a0 = fmaf(u.x, xv.x, a0);
            a1 = fmaf(u.y, xv.y, a1);
            a0 = fmaf(u.z, xv.z, a0);
            a1 = fmaf(u.w, xv.w, a1);
          }
          const int row = rbeg + k;
          float sacc = warp_sum(a0 + a1) * scale;
          if (P.lm_flush) sacc = flush_small(sacc);
          if (P.lm_bias) sacc += __ldg(P.lm_bias + row);
          if (lane == 0) P.logits[row] = sacc;
          const unsigned long long key = amax_key(sacc, (unsigned)row);
          best = key > best ? key : best;
        }
        while (cur < nitems - 1) {
          if (cur >= 0) release(A, S, item + cur);
          ++cur;
          wait_slot(A, S, item + cur);
        }
        if (cur >= 0) release(A, S, item + cur);
        item += nitems;
        tmark(step, pi, 3);
        best = warp_max_u64(best);
        if (lane == 0) wbest[wid] = best;
        consumer_sync();
        if (*S.cabort) return;
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
        tmark(step, pi, 4);
        if (A.phase_ns && blockIdx.x == 0 && tid == 0) A.phase_ns[(size_t)step * (5 * L + 1) + pi] = global_ns();
        continue;
      }
      if (ph == kPhQkv) {
        if (blockIdx.x == 0)  // block/forward.rs:11-13 and :22-24 on this thread's elements
          for (int j = 0, i = tid; i < d; i += kMkConsumers, ++j) {
            const float v = raw[i];
            if (v != v) nan_flag(st, pos, l, kNanInput);
            const float nv = (v * scale) * pick(wreg, j);
            if (nv != nv) nan_flag(st, pos, l, kNanAttnNorm);
          }
        // this block's cached K/V rows for the attention split: every writer
        // of rows < pos fenced its row before publishing (a step or more ago)
        if (au >= 0 && tid == 0) {
          const int g = au % P.nkv, s = au / P.nkv, t0 = s * chunk;
          const int n = min(ctx, t0 + chunk) - t0;
          const int n_old = max(0, min(n, ctx - 1 - t0));
          const uint32_t bytes = uint32_t(n_old) * hd * 4;
          fence_acq_rel_gpu();
          asm volatile("fence.proxy.async.global;" ::: "memory");
          *S.kv_armed = *S.kv_armed + 1;
          mbar_expect_tx(S.kv_bar, 2 * bytes);
          if (bytes) {
            bulk_g2s(S.kvbuf, Lw.kc + ((size_t)g * P.max_ctx + t0) * hd, bytes, S.kv_bar);
            bulk_g2s(S.kvbuf + (size_t)cap * hd, Lw.vc + ((size_t)g * P.max_ctx + t0) * hd, bytes, S.kv_bar);
          }
        }
      }
      const bool gemv_here = ph == kPhQkv ? has_q : ph == kPhOproj ? has_o : ph == kPhGateup ? has_g : has_d;
      if (gemv_here) {
        const int ub = (int)blockIdx.x * gp.upc;  // this CTA's first unit of the phase
        unsigned long long* fr =
            A.trace_ns ? A.trace_ns + (((size_t)blockIdx.x * A.n_steps + step) * (5 * L + 1) + pi) * kMkTrace + 5
                       : nullptr;
        mk_gemv(A, S, gp, W, rpu, xs, xsum, item, fr, [&](int a, int r, float y0, float y1, bool has1) {
          if (ph == kPhQkv) {
            const int u = a + (r >> 1);
            y0 = flush_small(y0 * scale) + bsm[2 * (u - ub)];
            y1 = flush_small(y1 * scale) + bsm[2 * (u - ub) + 1];
            const int head = u / half, i = u - head * half;
            const int c0 = P.rope_split ? i : 2 * i;
            const int c1 = P.rope_split ? i + half : 2 * i + 1;
            if (head < P.nh + P.nkv) {  // RoPE: v0*cos - v1*sin, v0*sin + v1*cos
              const float2 cs = rope[i];
              const float o0 = y0 * cs.x - y1 * cs.y;
              const float o1 = y0 * cs.y + y1 * cs.x;
              y0 = o0;
              y1 = o1;
            }
            uint2* dst = head < P.nh ? A.ll.q + head * hd
                                     : A.ll.kv + (head - P.nh) * hd;  // k heads then v heads
            st_ll(dst + c0, y0, e_out);
            st_ll(dst + c1, y1, e_out);
          } else if (ph == kPhGateup) {
            const int u = a + (r >> 1);
            const float gv = flush_small(y0 * scale) + bsm[2 * (u - ub)];
            const float uv = flush_small(y1 * scale) + bsm[2 * (u - ub) + 1];
            if (uv != uv) nan_flag(st, pos, l, kNanUp);
            const float act = swiglu_balanced(gv, uv);
            if (act != act) nan_flag(st, pos, l, kNanFfnOut);
            st_ll(A.ll.act + u, act, e_out);
          } else {  // OPROJ, DOWN: rows a + r (+1) with the residual
            const int row = a + r;
            const float* xr = ph == kPhOproj ? S.xres[0] : S.xres[1];
            uint2* dst = ph == kPhOproj ? A.ll.xa : A.ll.xb;
            for (int k = 0; k < 2; ++k) {
              if (k == 1 && !has1) break;
              const float y = flush_small((k ? y1 : y0) * scale) + bsm[row + k - ub];
              if (ph == kPhDown && y != y) nan_flag(st, pos, l, kNanProjFfn);
              const float xn = xr[row + k] + y;
              if (ph == kPhDown && xn != xn) nan_flag(st, pos, l, kNanResidual);
              st_ll(dst + row + k, xn, e_out);
            }
          }
        });
        tmark(step, pi, 3);
        const int flo = ph == kPhQkv ? kFlQkv : ph == kPhOproj ? kFlXa : ph == kPhGateup ? kFlAct : kFlXb;
        mk_publish(A.ll.flags + flo * gridDim.x, e_out);
      }
      tmark(step, pi, 4);
      if (A.phase_ns && blockIdx.x == 0 && tid == 0) A.phase_ns[(size_t)step * (5 * L + 1) + pi] = global_ns();
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
  S.xsum = f;
  f += mk_round32(pl.xs_floats / 32);
  for (int k = 0; k < 2; ++k) {
    S.xres[k] = f;
    f += mk_round32(A.P.d);
  }
  S.qbuf = f;
  f += mk_round32(pl.qbuf_floats);
  S.ps = f;
  f += pl.ps_floats;
  S.kvbuf = f;
  f += 2 * (size_t)pl.attn_chunk_cap * hd;
  S.part = f;
  f += kMkPartFloats;
  S.rope = reinterpret_cast<float2*>(f);
  f += 2 * hd;
  S.bias = f;
  f += 2 * pl.bias_floats;
  {  // the LayerW table: every phase reads its pointers and shapes from here
    unsigned char* lb = reinterpret_cast<unsigned char*>(f);
    const uint32_t* src = reinterpret_cast<const uint32_t*>(A.layers);
    uint32_t* dst = reinterpret_cast<uint32_t*>(lb);
    const int words = A.P.n_layers * int(sizeof(LayerW) / 4);
    for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
    S.layers = reinterpret_cast<const LayerW*>(lb);
    S.slots = lb + pl.layers_bytes;
  }
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
