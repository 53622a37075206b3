// fused.cuh -- persistent batch-1 decode with two exchanges per block.
//
// The same step as k_decode_mega (GenomicLLM::forward_core,
// src/nn/llm/forward.rs:7-63), restructured so that each transformer block
// costs two all-to-all exchanges instead of five.  The five-exchange kernel
// is latency-bound: every exchange through L2 costs 1.5-2.5 us of flag
// latency plus a gather, and a 24-block model pays 121 of them per token.
//
// Per block l, with R the residual stream entering the block:
//
//   phase A  (the attention half)
//     KV CTAs (2 * n_kv): attn_norm(R) -> this position's k (RoPE) or v rows
//       of one KV head -> LL words for the attention CTAs + the cache row.
//     attention CTAs (n_head * S): attn_norm(R) -> the q rows of one head
//       (RoPE) -> split-K attention over 1/S of the cached positions (the
//       last split also takes this position's k/v row) -> unnormalised
//       output O_s with its (max m_s, sum l_s) -> the head's attn_output
//       columns times O_s (a d-vector) -> after reading the (m, l) of the
//       head's other splits, scaled by exp(m_s - M) / (L + 1e-12) and added
//       into the accumulator YA with red.global.add.
//   phase B  (the FFN half), every CTA with ffn K-blocks (32 SwiGLU outputs
//     each): x_a = R + flush(YA) (+ bias); ffn_norm(x_a) -> its gate/up row
//     pairs -> SwiGLU -> the ffn_down columns of those K-blocks times the 32
//     outputs (a d-vector) -> red.global.add into YB.
//   R' = x_a + flush(YB) (+ bias): every CTA forms it from the two sums.
//
// Because the attention output projection and the down projection are
// linear, their inputs never have to be gathered: each CTA adds its
// contribution to the d-vector sums, and the reference's |y| < 1e-6 flush
// (genomic.rs:331-335) and bias are applied by the readers to the complete
// sums.  The float sums are accumulated in arrival order, so results vary
// from run to run at the rounding level (the parity bar is a tolerance).
//
// Exchanges: a CTA that finished its additions adds 1 to the phase's counter
// with release semantics (after a barrier); a reader polls the counter until
// every writer of the phase so far has added, loads it once with acquire
// semantics, and reads the sums with L2 loads.  The (m, l) pairs of the
// attention splits and this position's k/v rows travel as LL words ({value,
// epoch}, self-validating).  The sums are double-buffered by block parity and
// cleared by the attention CTAs two phases after their last read (every reader
// of a buffer has published to a counter the clearing CTA waited for).
//
// Weights stream through a shared-memory ring (lane 0 of warp 15 is the
// producer, 1-D TMA bulk copies, full/empty mbarriers) in this CTA's item
// order: per block its q (or k/v) rows, its attn_output column blocks, then
// per ffn K-block its gate/up rows and its ffn_down column block; then its
// lm_head rows (f32, or for a Q8_0 lm_head the int8 codes and f16 scales of
// each row, dequantised in the dot: 3.7x fewer bytes than the f32 rows).  attn_output and ffn_down are kept a second time K-block
// major (qsT[kb][row]) so that a CTA's columns are one contiguous run.  The
// cached K/V rows of a split are fetched by TMA while the CTA waits for its
// input.  Every wait is bounded (c_wait_ns) and reported as DevState::err.
#pragma once

#include "megakernel.cuh"

namespace gaje {

constexpr int kFuThreads = 512;
constexpr int kFuConsumerWarps = 15;
constexpr int kFuConsumers = kFuConsumerWarps * 32;
constexpr int kFuMaxSlots = 8;
constexpr int kFuHeader = 1024;
constexpr int kFuMaxSplits = 16;

// attn_output and ffn_down of a block, K-block major: qs[kb][row], sm[kb][row].
struct FuLayer {
  const uint4* wo_qs;
  const uint32_t* wo_sm;
  const uint4* dn_qs;
  const uint32_t* dn_sm;
};

struct FusedPlan {
  int S;          // attention splits per q head
  int nA;         // attention CTAs: n_head * S (CTAs [0, nA))
  int nKV;        // k/v CTAs: 2 * n_kv * kv_split (CTAs [nA, nA + nKV))
  int kv_split;   // CTAs per k or v head, each hd / kv_split of its rows
  int cap;        // K/V rows one split holds: cached chunk + this position's row
  int nslots;
  unsigned slot_bytes;
  int lm_rows_per_cta, lm_stage_rows;
  int ob_max;     // SwiGLU outputs of the busiest CTA
  int cb_max;     // ffn_down column blocks one CTA's outputs touch, at most
  int pv_groups;  // position groups of the P*V partial sums
};

struct FusedArgs {
  StepParams P;
  const LayerW* layers;
  const FuLayer* fl;
  FusedPlan plan;
  float* ya;      // [2][d] attention-projection sums
  float* yb;      // [2][d] down-projection sums
  unsigned* cnt;  // [2]: attention-half and FFN-half phase counters (zero at launch)
  uint2* kvnew;   // [2][nkv][hd] this position's k (rotated) and v rows
  uint2* mlx;     // [nh][S][2] (m, l) of every split
  uint2* tok;     // [1] the step's argmax
  unsigned epoch0;
  int n_steps;
  unsigned long long* trace;  // optional [grid][n_steps][L+1][kFuTrace] stamps
  int withhold;  // diagnostic: this CTA raises no attention-half flag in block 0 of step 0 (-1: none)
};

// Trace points per block (phase A 0-8, 15-21, phase B 9-14) and for the
// lm_head (block index L: 0 entry, 1 input ready, 2 staged, 3 rows done, 4
// token out); slot 22 of step 0's block 0 holds the CTA's SM id.
constexpr int kFuTrace = 24;

// Trace stamps are SM cycle counts (clock64: fine-grained, but per SM); each
// CTA also records (globaltimer, clock64) anchor pairs at its start and end,
// in the lm_head row of step 0 (slots 22, 23) and of the last step (slots 20,
// 21), from which the host maps its cycles onto the global nanosecond clock.
__device__ __forceinline__ unsigned long long fu_tstamp() { return (unsigned long long)clock64(); }
// The trace buffer of an instantiation: compiled out (a constant null) unless TRACE.
template <bool TRACE>
__device__ __forceinline__ unsigned long long* fu_trace(const FusedArgs& A) { return TRACE ? A.trace : nullptr; }

__host__ __device__ inline unsigned fu_epoch(unsigned e0, int L, int step, int l, int ph) {
  return e0 + unsigned(step) * unsigned(2 * L + 1) + unsigned(2 * l + ph) + 1u;
}
// The FFN half of a block: CTA c computes the SwiGLU outputs [u0, u0 + n)
// (its 2n gate/up rows, contiguous in the pair-interleaved layout) and their
// share of ffn_down (the 1-3 column blocks the range touches, the outputs of
// other CTAs staged as zeros).  The counts differ by at most one across the
// CTAs, the larger ones on the last CTAs (those without attention work): one
// GEMV and one column pass per CTA, whatever ff / grid is.
__host__ __device__ inline void fu_outs(int ff, int grid, int c, int& u0, int& n) {
  const int base = ff / grid, extra = ff % grid, first_extra = grid - extra;
  n = base + (c >= first_extra ? 1 : 0);
  u0 = c * base + (c > first_extra ? c - first_extra : 0);
}
// Cached positions of split s when `cached` positions precede this one.  The
// last split also takes this position's row, which it has to wait for (the
// KV CTAs compute it in the same phase), so with more than one split it takes
// that row only and the others share the cached positions: its wait then
// overlaps their longer chunks instead of adding to a full one.
__host__ __device__ inline void fu_split(int cached, int S, int s, int& t0, int& n_old) {
  if (S > 1 && s == S - 1) {
    t0 = cached;
    n_old = 0;
    return;
  }
  const int P = S > 1 ? S - 1 : 1;
  const int chunk = (cached + P - 1) / P;
  t0 = s * chunk;
  n_old = max(0, min(chunk, cached - t0));
}

// Raw row dots of one row GEMV: the q / k / v rows of a head, or a CTA's gate/up rows.
__host__ __device__ inline size_t fu_raw_floats(const FusedPlan& p, int hd) {
  const int r = 2 * p.ob_max > hd ? 2 * p.ob_max : hd;
  return size_t(mk_round32(r));
}
__host__ __device__ inline size_t fu_pv_floats(const FusedPlan& p, int hd) {
  const size_t a = size_t(p.pv_groups) * hd;
  return a > size_t(kFuConsumers) ? a : size_t(kFuConsumers);
}

struct FuShared {
  uint64_t* full;
  uint64_t* empty;
  uint64_t* kv_bar;
  volatile int* abort_flag;
  volatile int* issued;
  volatile int* cabort;
  volatile int* kv_armed;
  volatile int* kv_waited;
  float* R;      // [d] residual stream entering the block
  float* XA;     // [d] x_a of the block
  float* xs;     // [d] staged (normed, pre-scaled, swizzled) row-GEMV input
  float* xsum;   // [d/32]
  float* qbuf;   // [hd]
  float* ps;     // [cap] scores, then exp
  float* kvbuf;  // [cap][hd] K, then [cap][hd] V
  float* pv;     // [pv_groups][hd]
  float* ost;    // [hd] staged O_s, [hd/32] sums after it
  float* ast;    // [cb_max*32] staged SwiGLU outputs of the CTA's column blocks, [cb_max] sums after them
  float* nw;     // [d] the norm weights of the next staging (prefetched)
  float* rb;     // [hd] RoPE (cos, sin) of the position, [hd] this CTA's q/k/v bias rows
  float* gub;    // [ob_max*2] gate/up bias rows of this CTA's outputs
  float* raw;    // [max(hd, 2*ob_max)] raw row dots of a row GEMV
  float* ycol;   // [d] column-GEMV accumulators (rows 4t..4t+3 owned by thread t)
  float* misc;   // 64 floats: reductions, coefficients
  unsigned char* slots;
};

__device__ __forceinline__ void fu_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kFuConsumers) : "memory"); }

__device__ __forceinline__ float ld_rlx(const float* p) {
  float v;
  asm volatile("ld.relaxed.gpu.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_rlx(float* p, float v) {
  asm volatile("st.relaxed.gpu.global.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// Sum (or max) over the consumer threads, the same value in every thread.
// `red` holds 16 floats; consecutive calls must alternate buffers.
__device__ __forceinline__ float fu_total(float v, float* red, bool is_max) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = is_max ? warp_max(v) : warp_sum(v);
  if (lane == 0) red[wid] = v;
  fu_sync();
  float t = red[0];
  for (int k = 1; k < kFuConsumerWarps; ++k) t = is_max ? fmaxf(t, red[k]) : t + red[k];
  return t;
}

// Phase counters: every CTA that finished a phase's global writes (red.add,
// stores) adds 1 to the phase's counter with release semantics; a reader polls
// the counter (one lane, relaxed loads, bounded) until it reaches the number of
// writers so far, then loads it once with acquire semantics, which synchronises
// with every writer's release (each add continues the release sequence of the
// ones before it).  The other consumer warps wait at a named barrier, which
// orders their reads after the acquire.  False (and the CTA's abort raised)
// when the count did not come in time.  The counters start at zero in every
// launch, so a target is (blocks so far) * (writers per block).
__device__ __forceinline__ unsigned ld_rlx_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_acq_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __noinline__ bool fu_gate(const unsigned* cnt, unsigned target, volatile int* cabort, DevState* st) {
  // the last consumer warp polls: thread 0 may still be busy with its
  // release add and the next K/V request when the gate is reached
  if ((threadIdx.x >> 5) == kFuConsumerWarps - 1) {
    if ((threadIdx.x & 31) == 0) {
      bool ok = true;
      if (int(ld_rlx_u32(cnt) - target) < 0) {
        const unsigned long long t0 = global_ns();
        while (int(ld_rlx_u32(cnt) - target) < 0) {
          if (global_ns() - t0 > c_wait_ns) {
            ok = false;
            break;
          }
        }
      }
      if (ok) (void)ld_acq_u32(cnt);
      else {
        flag_timeout(st, 20);
        *cabort = 1;
      }
    }
    __syncwarp();
    bar_arrive_n(3);
  } else {
    bar_sync_n(3);
  }
  return !*cabort;
}
// End of a phase whose global writes readers wait for: a consumer barrier,
// then thread 0 adds this CTA's 1 to the phase counter (release).
__device__ __forceinline__ void fu_publish(unsigned* cnt) {
  fu_sync();
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
}

// ----------------------------------------------------------- producer
struct FuItem {
  const void* a;
  const void* b;
  uint32_t na, nb;
};
// The i-th weight item of this CTA within one block (-1 past the last).
__device__ __forceinline__ bool fu_block_item(const FusedArgs& A, const LayerW& Lw, const FuLayer& F, int i,
                                              FuItem& it) {
  const StepParams& P = A.P;
  const FusedPlan& pl = A.plan;
  const int c = blockIdx.x, hd = P.hd, d = P.d;
  int k = i;
  const Q4View& Q = Lw.qkv;
  if (c < pl.nA + pl.nKV) {
    int row0, nr = hd;
    if (c < pl.nA) {
      row0 = (c / pl.S) * hd;
    } else {
      const int j = c - pl.nA, hv = j / pl.kv_split, sl = j - hv * pl.kv_split, kv = hv / P.nkv, g = hv - kv * P.nkv;
      nr = hd / pl.kv_split;
      row0 = (P.nh + kv * P.nkv + g) * hd + sl * nr;
    }
    if (k == 0) {
      it.a = Q.qs + (size_t)row0 * Q.nb;
      it.na = uint32_t(nr) * Q.nb * 16;
      it.b = Q.sm + (size_t)row0 * Q.nbp;
      it.nb = uint32_t(nr) * Q.nbp * 4;
      return true;
    }
    --k;
    if (c < pl.nA) {
      if (k == 0) {
        const int kb0 = (c / pl.S) * (hd / 32), n = hd / 32;
        it.a = F.wo_qs + (size_t)kb0 * d;
        it.na = uint32_t(n) * d * 16;
        it.b = F.wo_sm + (size_t)kb0 * d;
        it.nb = uint32_t(n) * d * 4;
        return true;
      }
      --k;
    }
  }
  int u0, n;
  fu_outs(P.ff, gridDim.x, c, u0, n);
  if (n == 0 || k >= 2) return false;
  if (k == 0) {  // gate/up rows of the CTA's SwiGLU outputs
    const Q4View& G = Lw.gate_up;
    it.a = G.qs + (size_t)(2 * u0) * G.nb;
    it.na = uint32_t(2 * n) * G.nb * 16;
    it.b = G.sm + (size_t)(2 * u0) * G.nbp;
    it.nb = uint32_t(2 * n) * G.nbp * 4;
  } else {  // the ffn_down column blocks the outputs touch
    const int kb0 = u0 / 32, nblk = (u0 + n - 1) / 32 - kb0 + 1;
    it.a = F.dn_qs + (size_t)kb0 * d;
    it.na = uint32_t(nblk) * d * 16;
    it.b = F.dn_sm + (size_t)kb0 * d;
    it.nb = uint32_t(nblk) * d * 4;
  }
  return true;
}

// Every weight byte (body and lm_head) is read once per step and the weights
// are far larger than L2, so the streams are loaded with an evict-first L2
// policy: they do not displace the lines that are reused (the exchange sums,
// LL words, the K/V cache rows): 517.4 -> 513.8 and 518.7 -> 515.0 us per
// step on two boxes.  (Holding part of the lm_head in L2 across steps with an
// evict-last policy was slower: 48 MB 514.8, 80 MB 517.5, 110 MB 524.2 us;
// loading the K/V rows evict-last did not help either.)
__device__ void fu_producer(const FusedArgs& A, const FuShared& S) {
  const StepParams& P = A.P;
  const FusedPlan& pl = A.plan;
  const int rbeg = blockIdx.x * pl.lm_rows_per_cta, rend = min(P.V, rbeg + pl.lm_rows_per_cta);
  const uint64_t pol = l2_policy_evict_first();
  const unsigned char* lm_base = P.lm_q8 ? P.lm_q8 : reinterpret_cast<const unsigned char*>(P.lm_head);
  int item = 0;
  for (int step = 0; step < A.n_steps; ++step) {
    for (int l = 0; l <= P.n_layers; ++l) {
      for (int i = 0;; ++i) {
        FuItem it{nullptr, nullptr, 0u, 0u};
        if (l < P.n_layers) {
          if (!fu_block_item(A, A.layers[l], A.fl[l], i, it)) break;
        } else {
          const int r = rbeg + i * pl.lm_stage_rows;
          if (r >= rend) break;
          it.a = lm_base + (size_t)r * P.lm_row_bytes;
          it.na = uint32_t(min(pl.lm_stage_rows, rend - r)) * uint32_t(P.lm_row_bytes);
        }
        const int slot = item % pl.nslots;
        if (item >= pl.nslots && !mbar_wait(S.empty + slot, ((item / pl.nslots) - 1) & 1)) {
          flag_timeout(P.st, 21);
          *S.abort_flag = 1;
          return;
        }
        if (*S.abort_flag || *S.cabort) return;
        unsigned char* dst = S.slots + (size_t)slot * pl.slot_bytes;
        mbar_expect_tx(S.full + slot, it.na + it.nb);
        bulk_g2s_hint(dst, it.a, it.na, S.full + slot, pol);
        if (it.nb) bulk_g2s_hint(dst + it.na, it.b, it.nb, S.full + slot, pol);
        ++item;
        *S.issued = item;
      }
    }
  }
}

// ----------------------------------------------------------- consumers
__device__ __forceinline__ const unsigned char* fu_wait_slot(const FusedArgs& A, const FuShared& S, int item) {
  const int slot = item % A.plan.nslots;
  if (!*S.cabort && !*S.abort_flag && !mbar_wait(S.full + slot, (item / A.plan.nslots) & 1)) {
    flag_timeout(A.P.st, 22);
    *S.cabort = 1;
  }
  if (*S.abort_flag) *S.cabort = 1;
  return S.slots + (size_t)slot * A.plan.slot_bytes;
}
__device__ __forceinline__ void fu_release(const FusedArgs& A, const FuShared& S, int item) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(S.empty + item % A.plan.nslots);
}

// Raw dots of the nr rows of a row-major Q4 item against the staged xs, into
// out[nr] (shared memory).  Thread t takes row t / SL and the blocks
// t % SL, t % SL + SL, ... of it (SL slices per row, as many as the consumer
// threads allow), into part[]; then a thread per row adds its SL slices in
// order.  Independent blocks per thread keep the issue slots busy (a warp per
// row pair with a shuffle reduction measured 1.3x slower for 64 rows).
__device__ __forceinline__ void fu_rows_raw(const unsigned char* slot, int nr, int nb, int nbp, const float* xs,
                                         const float* xsum, float* part, float* out) {
  const int t = threadIdx.x;
  const int SL = max(1, min(nb, kFuConsumers / nr));
  const uint4* qs = reinterpret_cast<const uint4*>(slot);
  const uint32_t* sm = reinterpret_cast<const uint32_t*>(slot + (size_t)nr * nb * 16);
  if (t < nr * SL) {
    const int r = t / SL, c = t - r * SL;
    float acc = 0.f;
#pragma unroll 1
    for (int b = c; b < nb; b += SL) {
      float A0, A1, sc, mn;
      const uint4 q = qs[(size_t)r * nb + b];
      q4_pair_qx(q, q, false, xs, b, A0, A1);
      unpack_sm(sm[(size_t)r * nbp + b], sc, mn);
      acc = fmaf(sc, A0, fmaf(mn, xsum[b], acc));
    }
    part[t] = acc;
  }
  fu_sync();
  if (t < nr) {
    float s = 0.f;
    for (int c = 0; c < SL; ++c) s += part[t * SL + c];
    out[t] = s;
  }
}

// ycol[2p], ycol[2p+1] (+)= the raw dots of rows 2p, 2p+1 over nkb
// K-block-major column blocks against the staged xst / xsum (local block
// index), a thread per row pair (pairs p = tid, tid + 480, ...); init starts
// the accumulators at zero.
__device__ __forceinline__ void fu_cols(const unsigned char* slot, int d, int nkb, const float* xst, const float* xsum,
                                     float* ycol, bool init) {
  const uint4* qs = reinterpret_cast<const uint4*>(slot);
  const uint32_t* sm = reinterpret_cast<const uint32_t*>(slot + (size_t)nkb * d * 16);
#pragma unroll 1
  for (int p = threadIdx.x; p < d / 2; p += kFuConsumers) {
    float2 y = init ? make_float2(0.f, 0.f) : reinterpret_cast<const float2*>(ycol)[p];
#pragma unroll 1
    for (int kb = 0; kb < nkb; ++kb) {
      const uint4* q = qs + (size_t)kb * d + 2 * p;
      const uint2 s2 = *reinterpret_cast<const uint2*>(sm + (size_t)kb * d + 2 * p);
      const float xb = xsum[kb];
      float A0, A1, sc, mn;
      q4_pair_qx(q[0], q[1], true, xst, kb, A0, A1);
      unpack_sm(s2.x, sc, mn);
      y.x = fmaf(sc, A0, fmaf(mn, xb, y.x));
      unpack_sm(s2.y, sc, mn);
      y.y = fmaf(sc, A1, fmaf(mn, xb, y.y));
    }
    reinterpret_cast<float2*>(ycol)[p] = y;
  }
}
__device__ __forceinline__ void red_add2(float* p, float a, float b) {
  asm volatile("red.relaxed.gpu.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(a), "f"(b) : "memory");
}

// The cached K/V rows split s of a head of KV group g reads when `cached`
// positions precede this one: their first element in the group's cache and
// their bytes per cache.
__device__ __forceinline__ void fu_kv_span(const FusedArgs& A, int g, int s, int cached, size_t& row0,
                                           uint32_t& bytes) {
  int t0, n_old;
  fu_split(cached, A.plan.S, s, t0, n_old);
  row0 = ((size_t)g * A.P.max_ctx + t0) * A.P.hd;
  bytes = uint32_t(n_old) * A.P.hd * 4;
}
// Issues the TMA copies of a split's cached K/V rows of block l (a span of
// fu_kv_span; thread 0 of the consumers).
__device__ __forceinline__ void fu_kv_prefetch(const FusedArgs& A, const FuShared& S, int l, size_t row0,
                                               uint32_t bytes) {
  const LayerW& Lw = A.layers[l];
  // the rows were written by the KV CTAs of earlier blocks, and this thread
  // has acquired them since (its gate's fence): a proxy fence is enough to
  // hand them to the asynchronous (TMA) reads
  asm volatile("fence.proxy.async.global;" ::: "memory");
  *S.kv_armed = *S.kv_armed + 1;
  mbar_expect_tx(S.kv_bar, 2 * bytes);
  if (bytes) {
    bulk_g2s(S.kvbuf, Lw.kc + row0, bytes, S.kv_bar);
    bulk_g2s(S.kvbuf + (size_t)A.plan.cap * A.P.hd, Lw.vc + row0, bytes, S.kv_bar);
  }
}

// dst = base + flush(sum) + bias for this thread's elements (sum read from L2
// after an acquiring gate).  With nan_layer >= 0 (one CTA) the down
// projection's NaN guards of block/forward.rs:128-140 are raised.
__device__ __forceinline__ void fu_add_sum(float* dst, const float* base, const float* sum, const float* bias, int d,
                                        DevState* st, unsigned pos, int nan_layer) {
#pragma unroll 1
  for (int i0 = threadIdx.x; i0 < d; i0 += 2 * kFuConsumers) {
    const int i1 = i0 + kFuConsumers;
    const float s0 = __ldcg(sum + i0), s1 = i1 < d ? __ldcg(sum + i1) : 0.f;
    const float b0 = bias ? __ldg(bias + i0) : 0.f, b1 = (bias && i1 < d) ? __ldg(bias + i1) : 0.f;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = k ? i1 : i0;
      if (i >= d) break;
      const float y = flush_small(k ? s1 : s0) + (k ? b1 : b0);
      const float v = base[i] + y;
      if (nan_layer >= 0) {
        if (y != y) nan_flag(st, pos, nan_layer, kNanProjFfn);
        if (v != v) nan_flag(st, pos, nan_layer, kNanResidual);
      }
      dst[i] = v;
    }
  }
}

// The block-input and normed-output NaN guards of block/forward.rs:11-13,
// :22-24 over this thread's elements.  Out of line: it only runs when one of
// them can fire.
__device__ __noinline__ void fu_norm_guard(const float* x, const float* nw, int d, float inv, DevState* st,
                                           unsigned pos, int layer) {
  for (int i = threadIdx.x; i < d; i += kFuConsumers) {
    const float v = x[i];
    if (v != v) nan_flag(st, pos, layer, kNanInput);
    const float nv = (v * inv) * nw[i];
    if (nv != nv) nan_flag(st, pos, layer, kNanAttnNorm);
  }
}

// Stages x * nw into xs/xsum for the row GEMVs and returns 1/rms of x (the
// scale of the finished row dots), with the NaN guards when guard.  An input
// or normed output of this thread can only be NaN when the sum of squares or
// 1/rms is not finite (a non-finite x makes it so) or one of its norm weights
// is not: otherwise |x * inv| <= sqrt(d) and the product with a finite weight
// is a number, so the element checks are skipped.
__device__ __forceinline__ float fu_stage_norm(const float* x, const float* nw, int d, float eps, float* xs,
                                            float* xsum, float* red, bool guard, DevState* st, unsigned pos,
                                            int layer) {
  float ss = 0.f;
  bool wbad = false;
  const int lane = threadIdx.x & 31;
  // two elements per pass (whole warps: d % 32 == 0), their block sums'
  // shuffles interleaved
#pragma unroll 1
  for (int i0 = threadIdx.x; i0 < d; i0 += 2 * kFuConsumers) {
    const int i1 = i0 + kFuConsumers;
    const bool h1 = i1 < d;  // warp-uniform
    const float v0 = x[i0], w0 = nw[i0], v1 = h1 ? x[i1] : 0.f, w1 = h1 ? nw[i1] : 0.f;
    ss = fmaf(v0, v0, ss);
    if (h1) ss = fmaf(v1, v1, ss);
    wbad |= !(fabsf(w0) <= 3.402823466e38f) || !(fabsf(w1) <= 3.402823466e38f);
    float s0 = v0 * w0, s1 = v1 * w1;
    xs[swz(i0)] = s0 * nib_prescale(i0 & 7);
    if (h1) xs[swz(i1)] = s1 * nib_prescale(i1 & 7);
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    }
    if (lane == 0) {
      xsum[i0 >> 5] = s0;
      if (h1) xsum[i1 >> 5] = s1;
    }
  }
  const float tot = fu_total(ss, red, false);
  const float inv = 1.0f / sqrtf(tot / (float)d + eps);
  if (guard && (wbad || !(tot <= 3.402823466e38f) || !(inv <= 3.402823466e38f)))
    fu_norm_guard(x, nw, d, inv, st, pos, layer);
  return inv;
}

// The step's token: DevState::token for the first step of a launch, else the
// previous step's LL token word.
__device__ __forceinline__ bool fu_token(const FusedArgs& A, int step, unsigned& tok) {
  if (step == 0) {
    tok = __ldcg(&A.P.st->token);
    return true;
  }
  const unsigned e = fu_epoch(A.epoch0, A.P.n_layers, step - 1, A.P.n_layers, 0);
  uint2 w = ld_ll(A.tok);
  unsigned long long t0 = 0;
  while (w.y != e) {
    const unsigned long long t = global_ns();
    if (!t0) t0 = t;
    else if (t - t0 > c_wait_ns) return false;
    w = ld_ll(A.tok);
  }
  tok = w.x;
  return true;
}

// Loads n floats of global memory into shared memory (zeros without src).
__device__ __forceinline__ void fu_prefetch(float* dst, const float* src, int n) {
#pragma unroll 1
  for (int i0 = threadIdx.x; i0 < n; i0 += 2 * kFuConsumers) {  // both loads in flight together
    const int i1 = i0 + kFuConsumers;
    const float a = src ? __ldg(src + i0) : 0.f, b = (src && i1 < n) ? __ldg(src + i1) : 0.f;
    dst[i0] = a;
    if (i1 < n) dst[i1] = b;
  }
}

// The attention of split sp of head h at position pos (q in S.qbuf), by one
// warp (the caller's warp 0; no CTA barrier inside): the cached rows landed by
// TMA, this position's k/v row (LL words) for the last split, scores,
// softmax, (m, l) published, P*V, O staged for the output projection.  Lane
// l owns dims l, l+32, ... of q, k and v.  Scores go 32 positions at a time:
// each lane forms its partial dot for every position of the group and one
// butterfly reduce-scatter leaves position i's dot in lane i.  Returns the
// split's position count, or -1 when a wait ran out (the CTA's abort raised).
template <int VEC, bool TRACE>
__device__ __forceinline__ int fu_attend_warp(const FusedArgs& A, const FuShared& S, int l, int step, unsigned pos,
                                              int h, int sp, unsigned eA, uint32_t kv_bytes) {
  const StepParams& P = A.P;
  const FusedPlan& pl = A.plan;
  DevState* st = P.st;
  constexpr int HD = 32 * VEC;
  const int lane = threadIdx.x & 31, L = P.n_layers;
  unsigned long long* const tr = fu_trace<TRACE>(A);
  unsigned long long* trow = tr ? tr + (((size_t)blockIdx.x * A.n_steps + step) * (L + 1) + l) * kFuTrace : nullptr;
  if (trow && lane == 0) trow[16] = fu_tstamp();  // trace point 16: the split's attention starts
  const int n_old = int(kv_bytes / (HD * 4));  // the split's cached rows (fu_kv_span at this position)
  const bool last = sp == pl.S - 1;
  const int n = n_old + (last ? 1 : 0);
  float* Ks = S.kvbuf;
  float* Vs = S.kvbuf + (size_t)pl.cap * HD;
  const int g = h / (P.nh / P.nkv);
  bool ok = true;
  if (last) {  // this position's k and v rows: LL words of the KV CTAs
    const uint2* src = A.kvnew + (size_t)g * HD;
    const uint2* srcv = A.kvnew + (size_t)(P.nkv + g) * HD;
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      const int e = lane + 32 * v;
      uint2 wk = ld_ll(src + e), wv = ld_ll(srcv + e);
      unsigned long long tw = 0;
      while (wk.y != eA || wv.y != eA) {
        const unsigned long long t = global_ns();
        if (!tw) tw = t;
        else if (t - tw > c_wait_ns) {
          ok = false;
          break;
        }
        wk = ld_ll(src + e);
        wv = ld_ll(srcv + e);
      }
      Ks[(size_t)n_old * HD + e] = __uint_as_float(wk.x);
      Vs[(size_t)n_old * HD + e] = __uint_as_float(wv.x);
    }
  }
  const int use = *S.kv_waited;
  if (ok && !mbar_wait(S.kv_bar, use & 1)) ok = false;
  if (!__all_sync(0xffffffffu, ok)) {
    if (lane == 0) {
      flag_timeout(st, 24);
      *S.cabort = 1;
    }
    return -1;
  }
  __syncwarp();
  if (lane == 0) {
    *S.kv_waited = use + 1;
    if (trow) trow[4] = fu_tstamp();  // trace point 4: this split's K/V rows landed
  }
  // Scores, a lane per position: lane i of group g0 forms dot(q, K[g0 + i]) over
  // float4 columns visited in the rotated order (j + i) mod HD/4, so that any 8
  // consecutive lanes touch 8 distinct 16-byte bank groups of K and of q (no
  // bank conflict).  A rolled loop: far less code than the unrolled
  // 32-position butterfly it replaced, for the same arithmetic.
  constexpr int H4 = HD / 4;
  const float4* q4 = reinterpret_cast<const float4*>(S.qbuf);
  float m = -INFINITY;
  for (int g0 = 0; g0 < n; g0 += 32) {
    const int t = g0 + lane;
    if (t < n) {
      const float4* kr = reinterpret_cast<const float4*>(Ks + (size_t)t * HD);
      float a0 = 0.f, a1 = 0.f;
#pragma unroll 4
      for (int j = 0; j < H4; ++j) {
        const int jj = (j + lane) & (H4 - 1);
        const float4 kv = kr[jj], qv = q4[jj];
        a0 = fmaf(qv.x, kv.x, a0);
        a1 = fmaf(qv.y, kv.y, a1);
        a0 = fmaf(qv.z, kv.z, a0);
        a1 = fmaf(qv.w, kv.w, a1);
      }
      const float sc = (a0 + a1) * P.attn_scale;
      S.ps[t] = sc;
      m = fmaxf(m, sc);
    }
  }
  if (trow && lane == 0) trow[17] = fu_tstamp();  // trace point 17: scores done
  m = warp_max(m);
  __syncwarp();
  float lsum = 0.f;
  for (int t = lane; t < n; t += 32) {
    const float e = expf(S.ps[t] - m);
    S.ps[t] = e;
    lsum += e;
  }
  lsum = warp_sum(lsum);
  __syncwarp();
  if (lane == 0) {
    S.misc[40] = m;
    if (n > 0) {  // (m, l) of this split
      uint2* ml = A.mlx + ((size_t)h * pl.S + sp) * 2;
      st_ll(ml, m, eA);
      st_ll(ml + 1, lsum, eA);
    }
    if (trow) trow[18] = fu_tstamp();  // trace point 18: softmax done, (m, l) published
  }
  float acc[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) acc[v] = 0.f;
#pragma unroll 4
  for (int t = 0; t < n; ++t) {
    const float p = S.ps[t];
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[v] = fmaf(p, Vs[(size_t)t * HD + lane + 32 * v], acc[v]);
  }
  __syncwarp();
  if (lane == 0 && trow) trow[19] = fu_tstamp();  // trace point 19: P*V done
#pragma unroll
  for (int v = 0; v < VEC; ++v) mk_stage_elem(S.ost, S.ost + HD, lane + 32 * v, acc[v]);
  return n;
}

// The split weight of this CTA's O_s: exp(m_s - M) / (sum_s exp(m_s - M) l_s
// + 1e-12) over the head's splits, from their LL (m, l) words (warp 0), into
// S.misc[32].
__device__ __forceinline__ void fu_split_weight(const FusedArgs& A, const FuShared& S, unsigned pos, int h, int n,
                                             unsigned eA) {
  const FusedPlan& pl = A.plan;
  const int lane = threadIdx.x & 31;
  const uint2* ml = A.mlx + (size_t)h * pl.S * 2;
  float ms = -INFINITY, ls = 0.f;
  bool good = true;
  if (lane < pl.S) {
    int t0s, nos;
    fu_split(int(pos), pl.S, lane, t0s, nos);
    if (nos + (lane == pl.S - 1 ? 1 : 0) > 0) {  // splits without positions publish nothing
      uint2 wm = ld_ll(ml + 2 * lane), wl = ld_ll(ml + 2 * lane + 1);
      unsigned long long tw = 0;
      while (wm.y != eA || wl.y != eA) {
        const unsigned long long t = global_ns();
        if (!tw) tw = t;
        else if (t - tw > c_wait_ns) {
          good = false;
          break;
        }
        wm = ld_ll(ml + 2 * lane);
        wl = ld_ll(ml + 2 * lane + 1);
      }
      ms = __uint_as_float(wm.x);
      ls = __uint_as_float(wl.x);
    }
  }
  if (!__all_sync(0xffffffffu, good) && lane == 0) {
    flag_timeout(A.P.st, 25);
    *S.cabort = 1;
  }
  const float M = warp_max(ms);
  float wsum = 0.f;
#pragma unroll 1
  for (int k = 0; k < pl.S; ++k) {  // split order
    const float mk = __shfl_sync(0xffffffffu, ms, k), lk = __shfl_sync(0xffffffffu, ls, k);
    if (mk > -INFINITY) wsum = fmaf(expf(mk - M), lk, wsum);
  }
  if (lane == 0) S.misc[32] = n > 0 ? expf(S.misc[40] - M) / (wsum + 1e-12f) : 0.f;
}

// output_norm + this CTA's lm_head rows (ring stages) + argmax; the last CTA
// to finish publishes the step's token.  Returns false on an abort.
template <bool TRACE>
__device__ __forceinline__ bool fu_lm(const FusedArgs& A, const FuShared& S, int step, unsigned pos, int* item_io,
                                   unsigned long long* trace_row) {
  const StepParams& P = A.P;
  const FusedPlan& pl = A.plan;
  DevState* st = P.st;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, c = blockIdx.x, d = P.d, L = P.n_layers;
  const int G = gridDim.x;
  __shared__ unsigned long long wbest[kFuConsumerWarps];
  __shared__ int is_last;
  fu_prefetch(S.nw, P.out_norm, d);
  if (trace_row && tid == 0) trace_row[0] = fu_tstamp();
  if (!fu_gate(A.cnt + 1, unsigned((step + 1) * L) * unsigned(G), S.cabort, st)) return false;
  if (trace_row && tid == 0) trace_row[1] = fu_tstamp();
  const int gl = step * L + L - 1;
  fu_add_sum(S.R, S.XA, A.yb + (gl & 1) * d, A.layers[L - 1].down.bias, d, st, pos, c == 0 ? L - 1 : -1);
  fu_sync();
  float ss = 0.f;
  for (int i = tid; i < d; i += kFuConsumers) {
    const float v = S.R[i];
    ss = fmaf(v, v, ss);
    S.xs[i] = v * S.nw[i];
  }
  const float scale = 1.0f / sqrtf(fu_total(ss, S.misc, false) / (float)d + P.eps);
  if (trace_row && tid == 0) trace_row[2] = fu_tstamp();
  const float4* x4 = reinterpret_cast<const float4*>(S.xs);
  const int K4 = d >> 2;
  unsigned long long best = 0ull;
  const int rbeg = c * pl.lm_rows_per_cta;
  const int nrows = max(0, min(P.V, rbeg + pl.lm_rows_per_cta) - rbeg);
  const int nitems = (nrows + pl.lm_stage_rows - 1) / pl.lm_stage_rows;
  const int item = *item_io;
  int cur = -1;
  const unsigned char* slot = nullptr;
#pragma unroll 1
  for (int k = wid; k < nrows; k += kFuConsumerWarps) {
    const int it = k / pl.lm_stage_rows;
    while (cur < it) {
      if (cur >= 0) fu_release(A, S, item + cur);
      ++cur;
      slot = fu_wait_slot(A, S, item + cur);
    }
    const unsigned char* rowp = slot + (size_t)(k - it * pl.lm_stage_rows) * P.lm_row_bytes;
    float a0 = 0.f, a1 = 0.f;
    if (P.lm_q8) {
      // Q8_0 row: element e is int8 q[e] times the f16 scale of its 32-block,
      // the f32 value q * scale of blocks.rs:44-48 (exact), in the f32 path's
      // order, so the logits equal those of the dequantised rows
      const uint32_t* q4w = reinterpret_cast<const uint32_t*>(rowp);
      const __half* sc = reinterpret_cast<const __half*>(rowp + d);
#pragma unroll 2
      for (int j = lane; j < K4; j += 32) {
        const uint32_t w = q4w[j];
        const float s = __half2float(sc[j >> 3]);
        const float4 xv = x4[j];
        a0 = fmaf(__fmul_rn(float(int8_t(w & 0xFFu)), s), xv.x, a0);
        a1 = fmaf(__fmul_rn(float(int8_t((w >> 8) & 0xFFu)), s), xv.y, a1);
        a0 = fmaf(__fmul_rn(float(int8_t((w >> 16) & 0xFFu)), s), xv.z, a0);
        a1 = fmaf(__fmul_rn(float(int8_t(w >> 24)), s), xv.w, a1);
      }
    } else {
      const float4* w4 = reinterpret_cast<const float4*>(rowp);
#pragma unroll 2
      for (int j = lane; j < K4; j += 32) {
        const float4 u = w4[j], xv = x4[j];
        a0 = fmaf(u.x, xv.x, a0);
        a1 = fmaf(u.y, xv.y, a1);
        a0 = fmaf(u.z, xv.z, a0);
        a1 = fmaf(u.w, xv.w, a1);
      }
    }
    const int row = rbeg + k;
    float v = warp_sum(a0 + a1) * scale;
    if (P.lm_flush) v = flush_small(v);
    if (P.lm_bias) v += __ldg(P.lm_bias + row);
    if (lane == 0) P.logits[row] = v;
    const unsigned long long key = amax_key(v, (unsigned)row);
    best = key > best ? key : best;
  }
  while (cur < nitems - 1) {
    if (cur >= 0) fu_release(A, S, item + cur);
    ++cur;
    fu_wait_slot(A, S, item + cur);
  }
  if (cur >= 0) fu_release(A, S, item + cur);
  *item_io = item + nitems;
  if (trace_row && tid == 0) trace_row[3] = fu_tstamp();
  best = warp_max_u64(best);
  if (lane == 0) wbest[wid] = best;
  fu_sync();
  if (*S.cabort) return false;
  if (tid == 0) {
    unsigned long long b = 0;
    for (int i = 0; i < kFuConsumerWarps; ++i) b = wbest[i] > b ? wbest[i] : b;
    P.amax_part[c] = b;
    __threadfence();
    is_last = (atomicAdd(P.amax_cnt, 1u) == unsigned(G) - 1u);
  }
  fu_sync();
  if (is_last) {
    __threadfence();
    unsigned long long b = 0;
    for (int i = tid; i < G; i += kFuConsumers) {
      const unsigned long long v = __ldcg(P.amax_part + i);
      b = v > b ? v : b;
    }
    b = warp_max_u64(b);
    if (lane == 0) wbest[wid] = b;
    fu_sync();
    if (tid == 0) {
      unsigned long long r = 0;
      for (int i = 0; i < kFuConsumerWarps; ++i) r = wbest[i] > r ? wbest[i] : r;
      const unsigned idx = amax_index(r);
      st->argmax = idx;
      st->token = idx;
      if (st->hist_len < P.hist_cap) P.tok_hist[st->hist_len] = idx;
      st->hist_len += 1u;
      st->pos = pos + 1u;
      *P.amax_cnt = 0u;
      fence_acq_rel_gpu();  // the state and the counter reset before the token word
      st_ll(A.tok, __uint_as_float(idx), fu_epoch(A.epoch0, L, step, L, 0));
    }
  }
  fu_sync();
  if (trace_row && tid == 0) trace_row[4] = fu_tstamp();
  return true;
}

template <int HD, bool TRACE>
__device__ void fu_consumer(const FusedArgs& A, const FuShared& S) {
  const StepParams& P = A.P;
  const FusedPlan& pl = A.plan;
  DevState* st = P.st;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, c = blockIdx.x;
  const int L = P.n_layers, d = P.d, hd = P.hd, half = hd >> 1, G = gridDim.x;
  const bool roleA = c < pl.nA, roleKV = !roleA && c < pl.nA + pl.nKV;
  const int h = roleA ? c / pl.S : 0, sp = roleA ? c - h * pl.S : 0;
  // a k/v CTA: slice kvs of the rows of k (kvk 0) or v head kvg
  const int kvj = roleKV ? c - pl.nA : 0, kvh = kvj / pl.kv_split, kvs = kvj - kvh * pl.kv_split;
  const int kvk = kvh / P.nkv, kvg = kvh - kvk * P.nkv;
  // this CTA's q/k/v rows [qrow0, qrow0 + nqr) (pair-interleaved storage) and
  // the head's RoPE pair of their first two
  const int nqr = roleA ? hd : hd / pl.kv_split;
  const int qrow0 = roleA ? h * hd : (P.nh + kvk * P.nkv + kvg) * hd + kvs * nqr;
  const int pbase = roleA ? 0 : kvs * (nqr >> 1);
  int fo0, nfo;  // this CTA's SwiGLU outputs [fo0, fo0 + nfo)
  fu_outs(P.ff, G, c, fo0, nfo);
  const int fkb0 = fo0 / 32, fnblk = nfo > 0 ? (fo0 + nfo - 1) / 32 - fkb0 + 1 : 0;
  unsigned* cntA = A.cnt;
  unsigned* cntB = A.cnt + 1;
  int item = 0;
  const unsigned pos0 = __ldcg(&st->pos);
  unsigned long long* const trace = fu_trace<TRACE>(A);
  auto fmark = [&](int step, int l, int k) {
    if (trace && tid == 0) trace[(((size_t)c * A.n_steps + step) * (L + 1) + l) * kFuTrace + k] = fu_tstamp();
  };
  // this split's cached K/V rows at this step's position (cur) and the next one's (nxt)
  const int kv_g = roleA ? h / (P.nh / P.nkv) : 0;
  size_t kv_row_cur = 0, kv_row_nxt = 0;
  uint32_t kv_b_cur = 0, kv_b_nxt = 0;
  if (roleA) fu_kv_span(A, kv_g, sp, int(pos0), kv_row_cur, kv_b_cur);
  if (roleA && tid == 0) fu_kv_prefetch(A, S, 0, kv_row_cur, kv_b_cur);  // step 0, block 0
  for (int step = 0; step < A.n_steps; ++step) {
    const unsigned pos = pos0 + unsigned(step);
    if (step > 0) {
      kv_row_cur = kv_row_nxt;
      kv_b_cur = kv_b_nxt;
    }
    if (roleA) fu_kv_span(A, kv_g, sp, int(pos) + 1, kv_row_nxt, kv_b_nxt);
    for (int l = 0; l < L; ++l) {
      const LayerW& Lw = A.layers[l];
      const Q4View& Q = Lw.qkv;
      const int gl = step * L + l;
      const unsigned eA = fu_epoch(A.epoch0, L, step, l, 0);
      float* ya = A.ya + (gl & 1) * d;
      float* yb = A.yb + (gl & 1) * d;
      const float* yb_prev = A.yb + ((gl + 1) & 1) * d;  // YB of block l-1
      const float* dn_bias_prev = l > 0 ? A.layers[l - 1].down.bias : nullptr;
      // ===================================================== block input R
      // every CTA: the step's embedding row, or the previous block's x_a plus
      // its down-projection sum once every CTA has added to it
      const bool roleAttn = roleA || roleKV;
      if (roleAttn) {
        fmark(step, l, 0);
        // constants of the attention half while the input is in flight
        fu_prefetch(S.nw, Lw.attn_norm, d);
#pragma unroll 1
        for (int i = tid; i < half; i += kFuConsumers)
          reinterpret_cast<float2*>(S.rb)[i] = __ldg(P.rope + (size_t)pos * half + i);
        fu_prefetch(S.rb + hd, Q.bias ? Q.bias + qrow0 : nullptr, nqr);
      }
      if (l == 0) {
        unsigned tok = 0;
        if (!fu_token(A, step, tok)) {
          flag_timeout(st, 23);
          *S.cabort = 1;
        }
        fu_sync();
        if (*S.cabort) return;
        const float* src = P.embd + (size_t)(tok % (unsigned)P.V) * d;  // get_row_core: row token % V
#pragma unroll 1
        for (int i = tid; i < d; i += kFuConsumers) S.R[i] = __ldg(src + i);
      } else {
        if (!fu_gate(cntB, unsigned(gl) * unsigned(G), S.cabort, st)) return;
        fmark(step, l, 21);
        fu_add_sum(S.R, S.XA, yb_prev, dn_bias_prev, d, st, pos, c == 0 ? l - 1 : -1);
      }
      if (!roleAttn) fu_sync();  // (the attention half has its own barrier after the clearing)
      // ============================================================ phase A
      if (roleAttn) {
        if (roleA) {  // clear the sums read two phases ago: YA of block l-1, YB of block l-2
          const int per = (d + pl.nA - 1) / pl.nA;
#pragma unroll 1
          for (int i = tid; i < per; i += kFuConsumers) {
            const int j = c * per + i;
            if (j < d) {
              st_rlx(A.ya + ((gl + 1) & 1) * d + j, 0.f);
              st_rlx(yb + j, 0.f);
            }
          }
        }
        if (L == 1 && roleA && tid == 0 && step > 0) fu_kv_prefetch(A, S, 0, kv_row_cur, kv_b_cur);
        fu_sync();
        fmark(step, l, 1);
        const float inv = fu_stage_norm(S.R, S.nw, d, P.eps, S.xs, S.xsum, S.misc, c == 0, st, pos, l);
        fmark(step, l, 2);
        const unsigned char* slot = fu_wait_slot(A, S, item);
        fu_sync();
        if (*S.cabort) return;
        fu_rows_raw(slot, nqr, Q.nb, Q.nbp, S.xs, S.xsum, S.pv, S.raw);
        fu_release(A, S, item++);
        fu_sync();
        // epilogue, a thread per row pair: flush, bias, RoPE (q, k)
        if (tid < (nqr >> 1)) {
          const int p = pbase + tid;  // the pair within the head
          float y0 = flush_small(S.raw[2 * tid] * inv) + S.rb[hd + 2 * tid];
          float y1 = flush_small(S.raw[2 * tid + 1] * inv) + S.rb[hd + 2 * tid + 1];
          if (roleA || kvk == 0) {  // RoPE: v0*cos - v1*sin, v0*sin + v1*cos
            const float cs = S.rb[2 * p], sn = S.rb[2 * p + 1];
            const float o0 = y0 * cs - y1 * sn, o1 = y0 * sn + y1 * cs;
            y0 = o0;
            y1 = o1;
          }
          const int c0 = P.rope_split ? p : 2 * p, c1 = P.rope_split ? p + half : 2 * p + 1;
          if (roleA) {
            S.qbuf[c0] = y0;
            S.qbuf[c1] = y1;
          } else {  // this position's k or v row: the cache row, and LL words for the last splits
            float* cache = (kvk ? Lw.vc : Lw.kc) + ((size_t)kvg * P.max_ctx + pos) * hd;
            uint2* dst = A.kvnew + (size_t)(kvk * P.nkv + kvg) * hd;
            cache[c0] = y0;
            cache[c1] = y1;
            st_ll(dst + c0, y0, eA);
            st_ll(dst + c1, y1, eA);
          }
        }
        fu_sync();
        fmark(step, l, 3);
        if (roleA) {
          if (wid == 0) {
            const int na = fu_attend_warp<HD / 32, TRACE>(A, S, l, step, pos, h, sp, eA, kv_b_cur);
            if (lane == 0) reinterpret_cast<int*>(S.misc)[41] = na;
          }
          fu_sync();
          const int n = reinterpret_cast<const int*>(S.misc)[41];
          if (n < 0 || *S.cabort) return;
          fmark(step, l, 5);
          const unsigned char* wslot = fu_wait_slot(A, S, item);
          fu_sync();
          if (*S.cabort) return;
          // the head's split weight, by the last warp: it has no rows of the
          // output projection when d/2 <= 448 (the weight overlaps the column
          // pass), else it takes its rows after the weight
          if (wid == kFuConsumerWarps - 1) fu_split_weight(A, S, pos, h, n, eA);
          if (n > 0) fu_cols(wslot, d, hd / 32, S.ost, S.ost + hd, S.ycol, true);
          fu_release(A, S, item++);
          fmark(step, l, 6);
          fmark(step, l, 15);
          fu_sync();
          if (*S.cabort) return;
          const float cf = S.misc[32];
          fmark(step, l, 7);
          if (n > 0) {
#pragma unroll 1
            for (int p = tid; p < d / 2; p += kFuConsumers) {
              const float2 y = reinterpret_cast<const float2*>(S.ycol)[p];
              red_add2(ya + 2 * p, cf * y.x, cf * y.y);
            }
          }
          if (c == A.withhold && l == 0 && step == 0) fu_sync();  // the readers' waits run out
          else fu_publish(cntA);
          // the K/V buffer is free: the next block's (or next step's) cached rows,
          // requested off the critical path while the FFN half waits
          if (tid == 0) {
            const bool same_step = l + 1 < L;
            if (same_step || (step + 1 < A.n_steps && L > 1))
              fu_kv_prefetch(A, S, same_step ? l + 1 : 0, same_step ? kv_row_cur : kv_row_nxt,
                             same_step ? kv_b_cur : kv_b_nxt);
            if (trace) trace[(((size_t)c * A.n_steps + step) * (L + 1) + l) * kFuTrace + 20] = fu_tstamp();
          }
          fmark(step, l, 8);
        }
      }
      // ============================================================ phase B
      fu_prefetch(S.nw, Lw.ffn_norm, d);
      if (nfo > 0) fu_prefetch(S.gub, Lw.gate_up.bias ? Lw.gate_up.bias + (size_t)fo0 * 2 : nullptr, nfo * 2);
      if (!fu_gate(cntA, unsigned(gl + 1) * unsigned(pl.nA), S.cabort, st)) return;
      fmark(step, l, 9);
      fu_add_sum(S.XA, S.R, ya, Lw.wo.bias, d, st, pos, -1);
      fu_sync();
      if (*S.cabort) return;
      fmark(step, l, 10);
      if (nfo > 0) {
        const float inv = fu_stage_norm(S.XA, S.nw, d, P.eps, S.xs, S.xsum, S.misc, false, st, pos, l);
        fmark(step, l, 11);
        const Q4View& Gu = Lw.gate_up;
        const unsigned char* gslot = fu_wait_slot(A, S, item);
        fu_sync();
        if (*S.cabort) return;
        fu_rows_raw(gslot, 2 * nfo, Gu.nb, Gu.nbp, S.xs, S.xsum, S.pv, S.raw);
        fu_release(A, S, item++);
        fu_sync();
        // SwiGLU of the outputs, staged over the column blocks (zeros for other CTAs' outputs)
        if (wid < fnblk) {
          const int e = wid * 32 + lane, j = fkb0 * 32 + e - fo0;  // j: this CTA's output index
          float a = 0.f;
          if (j >= 0 && j < nfo) {
            const float gv = flush_small(S.raw[2 * j] * inv) + S.gub[2 * j];
            const float uv = flush_small(S.raw[2 * j + 1] * inv) + S.gub[2 * j + 1];
            if (uv != uv) nan_flag(st, pos, l, kNanUp);
            a = swiglu_balanced(gv, uv);
            if (a != a) nan_flag(st, pos, l, kNanFfnOut);
          }
          mk_stage_elem(S.ast, S.ast + pl.cb_max * 32, e, a);
        }
        fmark(step, l, 12);
        const unsigned char* dslot = fu_wait_slot(A, S, item);
        fu_sync();
        if (*S.cabort) return;
        fu_cols(dslot, d, fnblk, S.ast, S.ast + pl.cb_max * 32, S.ycol, true);
        fu_release(A, S, item++);
        fmark(step, l, 13);
#pragma unroll 1
        for (int p = tid; p < d / 2; p += kFuConsumers) {
          const float2 y = reinterpret_cast<const float2*>(S.ycol)[p];
          red_add2(yb + 2 * p, y.x, y.y);
        }
      }
      fu_publish(cntB);
      fmark(step, l, 14);
    }
    // ================================================================ LM
    unsigned long long* trow = trace ? trace + (((size_t)c * A.n_steps + step) * (L + 1) + L) * kFuTrace : nullptr;
    if (!fu_lm<TRACE>(A, S, step, pos, &item, trow)) return;
  }
}

// One instantiation per head size (the split attention's lanes hold HD / 32
// dims each) and with or without the trace stamps: each launch runs only the
// code of its shapes, which keeps the per-block instruction working set small.
template <int HD, bool TRACE>
__global__ void __launch_bounds__(kFuThreads, 1) k_decode_fused(const __grid_constant__ FusedArgs A) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const FusedPlan& pl = A.plan;
  const int d = A.P.d, hd = A.P.hd;
  FuShared S;
  S.full = reinterpret_cast<uint64_t*>(smem_raw);
  S.empty = S.full + kFuMaxSlots;
  S.kv_bar = S.empty + kFuMaxSlots;
  S.abort_flag = reinterpret_cast<volatile int*>(S.kv_bar + 1);
  S.issued = S.abort_flag + 1;
  S.cabort = S.abort_flag + 2;
  S.kv_armed = S.abort_flag + 3;
  S.kv_waited = S.abort_flag + 4;
  float* f = reinterpret_cast<float*>(smem_raw + kFuHeader);
  S.R = f;
  f += d;
  S.XA = f;
  f += d;
  S.xs = f;
  f += d;
  S.xsum = f;
  f += mk_round32(d / 32);
  S.qbuf = f;
  f += hd;
  S.ps = f;
  f += mk_round32(pl.cap);
  S.kvbuf = f;
  f += 2 * (size_t)pl.cap * hd;
  S.pv = f;  // P*V partials, and the row-GEMV slice sums (at most kFuConsumers)
  f += fu_pv_floats(pl, hd);
  S.ost = f;
  f += hd + 32;
  S.ast = f;
  f += mk_round32(pl.cb_max * 33);
  S.nw = f;
  f += d;
  S.rb = f;
  f += 2 * hd;
  S.gub = f;
  f += mk_round32(pl.ob_max * 2);
  S.raw = f;
  f += fu_raw_floats(pl, hd);
  S.ycol = f;
  f += d;
  S.misc = f;
  f += 64;
  S.slots = reinterpret_cast<unsigned char*>(f);
  if (threadIdx.x == 0) {
    for (int i = 0; i < pl.nslots; ++i) {
      mbar_init(S.full + i, 1);
      mbar_init(S.empty + i, kFuConsumerWarps);
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
  if (threadIdx.x >= kFuConsumers) {
    if (threadIdx.x == kFuConsumers) {
      fu_producer(A, S);
      const int issued = *S.issued;  // every issued copy lands before the CTA exits
      for (int it = max(0, issued - pl.nslots); it < issued; ++it)
        mbar_wait(S.full + it % pl.nslots, (it / pl.nslots) & 1);
    }
    return;
  }
  unsigned long long* const trace = fu_trace<TRACE>(A);
  unsigned long long* anchor =
      trace ? trace + (((size_t)blockIdx.x * A.n_steps) * (A.P.n_layers + 1) + A.P.n_layers) * kFuTrace : nullptr;
  if (anchor && threadIdx.x == 0) {
    anchor[22] = global_ns();
    anchor[23] = fu_tstamp();
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    trace[((size_t)blockIdx.x * A.n_steps) * (A.P.n_layers + 1) * kFuTrace + 22] = smid;  // block 0 row of step 0
  }
  fu_consumer<HD, TRACE>(A, S);
  // a K/V copy may still be in flight (the last prefetch, or an abort): it must land first
  if (threadIdx.x == 0 && *S.kv_armed > *S.kv_waited) mbar_wait(S.kv_bar, (*S.kv_waited) & 1);
  if (anchor && threadIdx.x == 0) {
    unsigned long long* last = anchor + (size_t)(A.n_steps - 1) * (A.P.n_layers + 1) * kFuTrace;
    last[21] = fu_tstamp();
    last[20] = global_ns();
  }
}

// The instantiation for a head size (32, 64 or 128), with or without trace stamps.
using FusedKernel = void (*)(const FusedArgs);
inline FusedKernel fused_kernel(int hd, bool trace) {
  if (hd == 32) return trace ? k_decode_fused<32, true> : k_decode_fused<32, false>;
  if (hd == 64) return trace ? k_decode_fused<64, true> : k_decode_fused<64, false>;
  return trace ? k_decode_fused<128, true> : k_decode_fused<128, false>;
}

// Dynamic shared memory of the fused kernel.
__host__ __device__ inline size_t fused_smem_bytes(const FusedPlan& p, int d, int hd) {
  const size_t floats = size_t(3) * d + mk_round32(d / 32) + hd + mk_round32(p.cap) + size_t(2) * p.cap * hd +
                        fu_pv_floats(p, hd) + hd + 32 + mk_round32(p.cb_max * 33) + d + 2 * hd + mk_round32(p.ob_max * 2) +
                        fu_raw_floats(p, hd) + d + 64;
  return kFuHeader + floats * 4 + size_t(p.nslots) * p.slot_bytes;
}

// K-block-major copy of a row-major Q4 matrix: qsT[kb][row] = qs[row][kb],
// smT[kb][row] = sm[row][kb], rows ld apart (ld >= N; rows N..ld-1 are not
// written).
__global__ void k_q4_kbmajor(Q4View W, uint4* qsT, uint32_t* smT, int ld) {
  const size_t n = (size_t)W.N * W.nb;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int kb = int(i / W.N), row = int(i - (size_t)kb * W.N);
    qsT[(size_t)kb * ld + row] = W.qs[(size_t)row * W.nb + kb];
    smT[(size_t)kb * ld + row] = W.sm[(size_t)row * W.nbp + kb];
  }
}

}  // namespace gaje
