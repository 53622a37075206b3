// megakernel.cuh -- persistent batch-1 decode: every phase of every block of
// GenomicLLM::forward_core (src/nn/llm/forward.rs:7-63), for n consecutive
// greedy steps, in one cooperative launch of one CTA per SM.
//
// Phases of a step (grid barrier after each):
//   for each block l:  QKV (attn_norm + attn_qkv + RoPE + KV append)
//                      ATTN (split-K flash decode, last CTA per KV head combines)
//                      OPROJ (attn_output + residual)
//                      GATEUP (ffn_norm + ffn_gate_up + SwiGLU)
//                      DOWN (ffn_down + residual)
//   LM (output_norm + f32 lm_head + argmax; the last CTA advances the state)
//
// Warp roles: warps 0-14 compute ("consumers"); lane 0 of warp 15 is a
// producer that walks this CTA's static schedule of "items" -- the weight rows
// of each phase, the cached K/V rows of its attention split, the lm_head row
// stages -- and streams each item into a ring of shared-memory slots with 1-D
// TMA bulk copies (no multicast), full/empty mbarrier pairs per slot.  The
// producer never joins the grid barriers, so while the consumers wait at one
// it is already fetching the next phases' weights: DRAM latency hides behind
// barrier latency.
//
// Grid barriers: a monotonic counter in global memory (zeroed before each
// launch); thread 0 of each CTA does fence + atomicAdd, then spins with
// ld.acquire.gpu for at most kWaitNs.  Every wait in this kernel is bounded;
// a wait that runs out sets DevState::err, the CTA stops producing and
// consuming, drains its in-flight copies (bounded) and exits.
// Data written by other CTAs during the launch is read with ld.global.cg.
#pragma once

#include "kernels.cuh"

namespace gaje {

constexpr int kMkThreads = 512;
constexpr int kMkConsumerWarps = 15;
constexpr int kMkConsumers = kMkConsumerWarps * 32;
constexpr int kMkMaxSlots = 8;
constexpr int kMkHeader = 1024;      // mbarriers + flags
constexpr int kMkPartFloats = 1024;  // split-K partials / row sums
constexpr int kMkMaxVecPerThread = 20;  // activation loads per consumer thread (K <= 9600)

// Per-phase work split of a GEMV: units (rows or row pairs) per CTA, and units
// per slot-sized item.
struct MkGemv {
  int units, upc, units_per_item;
};

struct MegaPlan {
  int nslots;
  unsigned slot_bytes;
  MkGemv q, o, g, d;
  int lm_rows_per_cta, lm_stage_rows;
  int xs_floats;   // activation buffer capacity
  int ps_floats;   // attention score buffer capacity (G * chunk_max)
  int attn_chunk_cap;
};

struct MegaArgs {
  StepParams P;
  const LayerW* layers;     // [n_layers], device memory
  MegaPlan plan;
  unsigned* bar;            // grid barrier counter, zero at launch
  int n_steps;
  int block_k;              // block K-WTA k (0 = off)
  unsigned long long* phase_ns;  // optional [n_steps][5*L+1] phase end stamps (CTA 0)
};

__host__ __device__ inline size_t mega_smem_bytes(const MegaPlan& p) {
  return kMkHeader + size_t(p.xs_floats) * 4 + size_t(p.ps_floats) * 4 + size_t(kMkPartFloats) * 4 +
         size_t(p.nslots) * p.slot_bytes;
}

struct MkShared {
  uint64_t* full;
  uint64_t* empty;
  volatile int* abort_flag;  // raised by the producer (read by consumers only via cabort)
  volatile int* issued;      // items the producer has issued
  volatile int* cabort;      // consumers' abort decision: written before, read after a consumer barrier
  float* xs;
  float* ps;
  float* part;
  unsigned char* slots;
};

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kMkConsumers) : "memory"); }

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier for the consumer threads of every CTA.  Returns false (and
// raises the CTA's abort flag) if the wait ran out.
__device__ __forceinline__ bool grid_barrier(const MegaArgs& A, const MkShared& S, unsigned& target) {
  consumer_sync();
  target += gridDim.x;
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(A.bar, 1u);
    if (ld_acquire_u32(A.bar) < target) {
      const unsigned long long t0 = global_ns();
      while (ld_acquire_u32(A.bar) < target) {
        if (global_ns() - t0 > kWaitNs) {
          flag_timeout(A.P.st, 10);
          *S.cabort = 1;
          break;
        }
      }
    }
    if (*S.abort_flag) *S.cabort = 1;
  }
  consumer_sync();
  return *S.cabort == 0;
}

// ----------------------------------------------------------- the schedule
// Both roles enumerate the same items in the same order.  An item is one
// bulk-copy batch into one slot.
struct Item {
  const void* src0;
  const void* src1;
  uint32_t bytes0, bytes1;
  uint32_t dst1;  // byte offset of the second copy inside the slot
};

// GEMV item k of this CTA's rows for phase m: rows [row_a, row_b) of W.
__device__ __forceinline__ Item gemv_item(const Q4View& W, int rpu, int unit_a, int unit_b) {
  const int ra = unit_a * rpu, nr = (unit_b - unit_a) * rpu;
  Item it;
  it.src0 = W.qs + (size_t)ra * W.nb;
  it.bytes0 = uint32_t(nr) * W.nb * 16;
  it.src1 = W.sm + (size_t)ra * W.nbp;
  it.bytes1 = uint32_t(nr) * W.nbp * 4;
  it.dst1 = it.bytes0;
  return it;
}

__device__ __forceinline__ void cta_units(const MkGemv& g, int& u0, int& u1) {
  u0 = blockIdx.x * g.upc;
  u1 = min(g.units, u0 + g.upc);
  if (u0 > u1) u0 = u1;
}

// Splits per KV head in the persistent kernel: at most one (head, split) unit
// per CTA.
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
  auto issue = [&](const Item& it) {
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
    mbar_expect_tx(S.full + slot, it.bytes0 + it.bytes1);
    if (it.bytes0) bulk_g2s(dst, it.src0, it.bytes0, S.full + slot);
    if (it.bytes1) bulk_g2s(dst + it.dst1, it.src1, it.bytes1, S.full + slot);
    ++item;
    *S.issued = item;
  };
  const unsigned pos0 = __ldcg(&P.st->pos);
  const int G = P.nh / P.nkv;
  for (int step = 0; step < A.n_steps && ok; ++step) {
    const int ctx = int(pos0) + step + 1;
    for (int l = 0; l < P.n_layers && ok; ++l) {
      const LayerW& L = A.layers[l];
      const MkGemv* gs[4] = {&pl.q, &pl.o, &pl.g, &pl.d};
      const Q4View* ws[4] = {&L.qkv, &L.wo, &L.gate_up, &L.down};
      const int rpus[4] = {2, 1, 2, 1};
      for (int ph = 0; ph < 4 && ok; ++ph) {
        if (ph == 1) {  // attention K/V rows before OPROJ
          int nsplit, chunk;
          const int u = attn_unit(ctx, P.nkv, nsplit, chunk);
          if (u >= 0) {
            const int g = u % P.nkv, s = u / P.nkv, t0 = s * chunk;
            const int n = min(ctx, t0 + chunk) - t0;
            const int n_old = max(0, min(n, ctx - 1 - t0));
            Item it;
            it.src0 = L.kc + ((size_t)g * P.max_ctx + t0) * P.hd;
            it.src1 = L.vc + ((size_t)g * P.max_ctx + t0) * P.hd;
            it.bytes0 = it.bytes1 = uint32_t(n_old) * P.hd * 4;
            it.dst1 = uint32_t(pl.attn_chunk_cap) * P.hd * 4;
            // cache rows written earlier in this launch are read by TMA (async proxy)
            asm volatile("fence.proxy.async.global;" ::: "memory");
            issue(it);
          }
        }
        int u0, u1;
        cta_units(*gs[ph], u0, u1);
        for (int a = u0; a < u1 && ok; a += gs[ph]->units_per_item)
          issue(gemv_item(*ws[ph], rpus[ph], a, min(u1, a + gs[ph]->units_per_item)));
      }
    }
    // lm_head row stages
    const int rbeg = blockIdx.x * pl.lm_rows_per_cta;
    const int rend = min(P.V, rbeg + pl.lm_rows_per_cta);
    for (int r = rbeg; r < rend && ok; r += pl.lm_stage_rows) {
      const int rows = min(pl.lm_stage_rows, rend - r);
      Item it;
      it.src0 = P.lm_head + (size_t)r * P.d;
      it.bytes0 = uint32_t(rows) * P.d * 4;
      it.src1 = nullptr;
      it.bytes1 = 0;
      it.dst1 = 0;
      issue(it);
    }
    (void)G;
  }
}

// ----------------------------------------------------------- consumers
// Waits for item `item`'s slot; false (abort) if the wait ran out.
// Every consumer thread waits (bounded) on the slot's full barrier, then all
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

// Loads src[0..K) (written by other CTAs: L2-only loads, all issued before
// use) into swizzled smem; optional RMSNorm with weight w; returns NaN flags.
__device__ __forceinline__ void mk_load_vec(const float* src, int K, float* xs, const float* w, float eps,
                                            float* red, bool& nan_in, bool& nan_out, float scale_in = 1.0f) {
  const int tid = threadIdx.x;
  float v[kMkMaxVecPerThread];
#pragma unroll
  for (int k = 0; k < kMkMaxVecPerThread; ++k) {
    const int i = tid + k * kMkConsumers;
    v[k] = i < K ? __ldcg(src + i) : 0.f;
  }
  float ss = 0.f;
  int bad = 0;
#pragma unroll
  for (int k = 0; k < kMkMaxVecPerThread; ++k) {
    ss = fmaf(v[k], v[k], ss);
    bad |= (v[k] != v[k]);
  }
  nan_in = false;
  nan_out = false;
  if (w) {
    ss = warp_sum(ss);
    const int lane = tid & 31, wid = tid >> 5;
    if (lane == 0) {
      red[wid] = ss;
      red[32 + wid] = __int_as_float(bad);
    }
    consumer_sync();
    float t = lane < kMkConsumerWarps ? red[lane] : 0.f;
    int b = lane < kMkConsumerWarps ? __float_as_int(red[32 + lane]) : 0;
    t = warp_sum(t);
    b = __any_sync(0xffffffffu, b != 0);
    nan_in = b != 0;
    const float inv = 1.0f / sqrtf(t / (float)K + eps);
    int bo = 0;
#pragma unroll
    for (int k = 0; k < kMkMaxVecPerThread; ++k) {
      const int i = tid + k * kMkConsumers;
      if (i < K) {
        const float o = (v[k] * inv) * w[i];
        bo |= (o != o);
        xs[swz(i)] = o;
      }
    }
    consumer_sync();  // everyone has read red; xs complete
    if (lane == 0) red[64 + wid] = __int_as_float(bo);
    consumer_sync();
    int bb = lane < kMkConsumerWarps ? __float_as_int(red[64 + lane]) : 0;
    nan_out = __any_sync(0xffffffffu, bb != 0);
  } else {
#pragma unroll
    for (int k = 0; k < kMkMaxVecPerThread; ++k) {
      const int i = tid + k * kMkConsumers;
      if (i < K) xs[swz(i)] = scale_in != 1.0f ? v[k] * scale_in : v[k];
    }
    consumer_sync();
  }
}

// RMSNorm of the (swizzled) d-vector already in xs, in place.  With `plain`,
// the result is written unswizzled (element i at xs[i]) for the f32 rows.
__device__ __forceinline__ void mk_norm_smem(float* xs, int K, const float* w, float eps, float* red, bool plain,
                                             bool& nan_out) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  float v[kMkMaxVecPerThread];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMkMaxVecPerThread; ++k) {
    const int i = tid + k * kMkConsumers;
    v[k] = i < K ? xs[swz(i)] : 0.f;
    ss = fmaf(v[k], v[k], ss);
  }
  ss = warp_sum(ss);
  if (lane == 0) red[wid] = ss;
  consumer_sync();
  float t = lane < kMkConsumerWarps ? red[lane] : 0.f;
  t = warp_sum(t);
  const float inv = 1.0f / sqrtf(t / (float)K + eps);
  int bo = 0;
#pragma unroll
  for (int k = 0; k < kMkMaxVecPerThread; ++k) {
    const int i = tid + k * kMkConsumers;
    if (i < K) {
      const float o = (v[k] * inv) * w[i];
      bo |= (o != o);
      xs[plain ? i : swz(i)] = o;
    }
  }
  consumer_sync();
  if (lane == 0) red[64 + wid] = __int_as_float(bo);
  consumer_sync();
  const int bb = lane < kMkConsumerWarps ? __float_as_int(red[64 + lane]) : 0;
  nan_out = __any_sync(0xffffffffu, bb != 0);
}

// Rows [0, R) of one staged item: per-row sums (flushed + bias) into rowsum.
// Warps split rows; with fewer rows than warps a row's blocks are split
// across g warps (split-K) and reduced in a fixed order.
__device__ __forceinline__ void mk_rows(const unsigned char* slot, int R, int nb, int nbp, const float* xs,
                                        const float* bias, int row0, float* part, float* rowsum) {
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
        if (b < nb) acc += q4_block_dot(qs[(size_t)rr * nb + b], sm[(size_t)rr * nbp + b], xs, b);
      }
      acc = warp_sum(acc);
      if (lane == 0) part[rr * g + slice] = acc;
    }
  }
  consumer_sync();
  for (int t = threadIdx.x; t < R; t += kMkConsumers) {
    float s = 0.f;
    for (int k = 0; k < g; ++k) s += part[t * g + k];
    s = flush_small(s);
    if (bias) s += bias[row0 + t];
    rowsum[t] = s;
  }
  consumer_sync();
}

// CTA-local lateral_inhibition_kwta on the d-vector held (swizzled) in xs:
// exact k-th largest by radix select, values below become -1e9.  Writes the
// masked vector back to xs; CTA 0 also writes it to `out`.
__device__ void mk_block_kwta(float* xs, int d, int k, unsigned* hist, float* out) {
  const int tid = threadIdx.x;
  unsigned prefix = 0u, mask = 0u, kk = unsigned(k);
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kMkConsumers) hist[i] = 0u;
    consumer_sync();
    for (int i = tid; i < d; i += kMkConsumers) {
      const unsigned key = ord_key(xs[swz(i)]);
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
  for (int i = tid; i < d; i += kMkConsumers) {
    float v = xs[swz(i)];
    if (v < thr) v = -1e9f;
    xs[swz(i)] = v;
    if (out) out[i] = v;
  }
  consumer_sync();
}

__device__ void mk_consumer(const MegaArgs& A, const MkShared& S) {
  const StepParams& P = A.P;
  const MegaPlan& pl = A.plan;
  DevState* st = P.st;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  __shared__ float red[128];
  __shared__ unsigned hist[260];
  __shared__ unsigned long long wbest[32];
  __shared__ int is_last;
  __shared__ float mls[2 * kAttnMaxGroup];
  __shared__ float wsh[kAttnMaxGroup * kAttnMaxSplits];
  __shared__ float linv[kAttnMaxGroup];
  int item = 0;
  unsigned bar_target = 0;
  const unsigned pos0 = __ldcg(&st->pos);
  const int G = P.nh / P.nkv, hd = P.hd, half = hd >> 1;
  float* rowsum = S.part + 512;
  unsigned long long* stamp = A.phase_ns;
  const int stamps_per_step = 5 * P.n_layers + 1;
  auto mark = [&](int step, int k) {
    if (stamp && blockIdx.x == 0 && tid == 0) stamp[(size_t)step * stamps_per_step + k] = global_ns();
  };

  for (int step = 0; step < A.n_steps; ++step) {
    const unsigned pos = pos0 + step;
    const int ctx = int(pos) + 1;
    for (int l = 0; l < P.n_layers; ++l) {
      const LayerW& L = A.layers[l];
      bool nin, nout;
      // ------------------------------------------------ QKV
      {
        const float* src = P.x;
        if (l == 0) {
          const unsigned tok = __ldcg(&st->token) % (unsigned)P.V;
          src = P.embd + (size_t)tok * P.d;
        }
        if (A.block_k > 0 && l > 0) {
          // the previous block's K-WTA on x (block/forward.rs:145-149); NaN in
          // x was already reported by the previous block's residual guard
          mk_load_vec(src, P.d, S.xs, nullptr, 0.f, red, nin, nout);
          mk_block_kwta(S.xs, P.d, A.block_k, hist, blockIdx.x == 0 ? P.x : nullptr);
          mk_norm_smem(S.xs, P.d, L.attn_norm, P.eps, red, false, nout);
          nin = false;
        } else {
          mk_load_vec(src, P.d, S.xs, L.attn_norm, P.eps, red, nin, nout);
          if (l == 0 && blockIdx.x == 0)
            for (int i = tid; i < P.d; i += kMkConsumers) P.x[i] = __ldcg(src + i);
        }
        if (blockIdx.x == 0 && tid == 0) {
          if (nin) nan_flag(st, pos, l, kNanInput);
          if (nout) nan_flag(st, pos, l, kNanAttnNorm);
        }
        int u0, u1;
        cta_units(pl.q, u0, u1);
        for (int a = u0; a < u1; a += pl.q.units_per_item) {
          const int b = min(u1, a + pl.q.units_per_item);
          const unsigned char* slot = take(A, S, item);
          if (!slot) return;
          mk_rows(slot, (b - a) * 2, L.qkv.nb, L.qkv.nbp, S.xs, L.qkv.bias, a * 2, S.part, rowsum);
          for (int u = a + tid; u < b; u += kMkConsumers) {
            float y0 = rowsum[(u - a) * 2], y1 = rowsum[(u - a) * 2 + 1];
            const int head = u / half, i = u - head * half;
            const int c0 = P.rope_split ? i : 2 * i;
            const int c1 = P.rope_split ? i + half : 2 * i + 1;
            if (head < P.nh + P.nkv) {
              const float2 cs = P.rope[(size_t)pos * half + i];
              const float o0 = y0 * cs.x - y1 * cs.y;
              const float o1 = y0 * cs.y + y1 * cs.x;
              y0 = o0;
              y1 = o1;
            }
            if (head < P.nh) {
              P.q[head * hd + c0] = y0;
              P.q[head * hd + c1] = y1;
            } else {
              const bool is_k = head < P.nh + P.nkv;
              const int g = is_k ? head - P.nh : head - P.nh - P.nkv;
              float* c = (is_k ? L.kc : L.vc) + ((size_t)g * P.max_ctx + pos) * hd;
              c[c0] = y0;
              c[c1] = y1;
            }
          }
          release(A, S, item++);
        }
      }
      if (!grid_barrier(A, S, bar_target)) return;
      mark(step, 5 * l + 0);
      // ------------------------------------------------ ATTN
      {
        int nsplit, chunk;
        const int u = attn_unit(ctx, P.nkv, nsplit, chunk);
        if (u >= 0) {
          const int g = u % P.nkv, s = u / P.nkv, t0 = s * chunk;
          const int n = min(ctx, t0 + chunk) - t0;
          const int n_old = max(0, min(n, ctx - 1 - t0));
          const unsigned char* slot = take(A, S, item);
          if (!slot) return;
          float* Ks = reinterpret_cast<float*>(const_cast<unsigned char*>(slot));
          float* Vs = Ks + (size_t)pl.attn_chunk_cap * hd;
          float* qs = S.xs;  // q of the group's heads
          float* ps = S.ps;
          for (int i = tid; i < G * hd; i += kMkConsumers) qs[i] = __ldcg(P.q + (size_t)g * G * hd + i);
          if (n > n_old) {  // this step's own row, written in the QKV phase
            const float* kn = L.kc + ((size_t)g * P.max_ctx + t0 + n_old) * hd;
            const float* vn = L.vc + ((size_t)g * P.max_ctx + t0 + n_old) * hd;
            for (int i = tid; i < hd; i += kMkConsumers) {
              Ks[(size_t)n_old * hd + i] = __ldcg(kn + i);
              Vs[(size_t)n_old * hd + i] = __ldcg(vn + i);
            }
          }
          consumer_sync();
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
              const float e = expf(ps[j * chunk + t] - m);
              ps[j * chunk + t] = e;
              lsum += e;
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
          // the slot was written through the generic proxy (the new row)
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          release(A, S, item++);
          __threadfence();
          consumer_sync();
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
              P.attn[((size_t)g * G + j) * hd + e] = (O0 + O1) * linv[j];
            }
            if (tid == 0) P.attn_cnt[g] = 0u;
          }
        }
      }
      if (!grid_barrier(A, S, bar_target)) return;
      mark(step, 5 * l + 1);
      // ------------------------------------------------ OPROJ
      {
        mk_load_vec(P.attn, L.wo.K, S.xs, nullptr, 0.f, red, nin, nout);
        int u0, u1;
        cta_units(pl.o, u0, u1);
        for (int a = u0; a < u1; a += pl.o.units_per_item) {
          const int b = min(u1, a + pl.o.units_per_item);
          const unsigned char* slot = take(A, S, item);
          if (!slot) return;
          mk_rows(slot, b - a, L.wo.nb, L.wo.nbp, S.xs, L.wo.bias, a, S.part, rowsum);
          for (int r = a + tid; r < b; r += kMkConsumers) P.x[r] = __ldcg(P.x + r) + rowsum[r - a];
          release(A, S, item++);
        }
      }
      if (!grid_barrier(A, S, bar_target)) return;
      mark(step, 5 * l + 2);
      // ------------------------------------------------ GATEUP
      {
        mk_load_vec(P.x, P.d, S.xs, L.ffn_norm, P.eps, red, nin, nout);
        int u0, u1;
        cta_units(pl.g, u0, u1);
        for (int a = u0; a < u1; a += pl.g.units_per_item) {
          const int b = min(u1, a + pl.g.units_per_item);
          const unsigned char* slot = take(A, S, item);
          if (!slot) return;
          mk_rows(slot, (b - a) * 2, L.gate_up.nb, L.gate_up.nbp, S.xs, L.gate_up.bias, a * 2, S.part, rowsum);
          for (int u = a + tid; u < b; u += kMkConsumers) {
            const float gv = rowsum[(u - a) * 2], uv = rowsum[(u - a) * 2 + 1];
            if (uv != uv) nan_flag(st, pos, l, kNanUp);
            const float act = swiglu_balanced(gv, uv);
            if (act != act) nan_flag(st, pos, l, kNanFfnOut);
            P.act[u] = act;
          }
          release(A, S, item++);
        }
      }
      if (!grid_barrier(A, S, bar_target)) return;
      mark(step, 5 * l + 3);
      // ------------------------------------------------ DOWN
      {
        mk_load_vec(P.act, P.ff, S.xs, nullptr, 0.f, red, nin, nout);
        if (P.use_genomic_norm) {  // block/forward.rs:115-123, h_scale = 1
          float ss = 0.f;
          for (int i = tid; i < P.ff; i += kMkConsumers) {
            const float v = S.xs[i];
            ss = fmaf(v, v, ss);
          }
          ss = warp_sum(ss);
          if (lane == 0) red[wid] = ss;
          consumer_sync();
          float t = lane < kMkConsumerWarps ? red[lane] : 0.f;
          t = warp_sum(t);
          const float rms = sqrtf(t / (float)P.ff + P.eps);
          if (rms > 1.0f) {
            const float sc = 1.0f / rms;
            for (int i = tid; i < P.ff; i += kMkConsumers) S.xs[i] = S.xs[i] * sc;
          }
          consumer_sync();
        }
        int u0, u1;
        cta_units(pl.d, u0, u1);
        for (int a = u0; a < u1; a += pl.d.units_per_item) {
          const int b = min(u1, a + pl.d.units_per_item);
          const unsigned char* slot = take(A, S, item);
          if (!slot) return;
          mk_rows(slot, b - a, L.down.nb, L.down.nbp, S.xs, L.down.bias, a, S.part, rowsum);
          for (int r = a + tid; r < b; r += kMkConsumers) {
            const float y = rowsum[r - a];
            if (y != y) nan_flag(st, pos, l, kNanProjFfn);
            const float xn = __ldcg(P.x + r) + y;
            if (xn != xn) nan_flag(st, pos, l, kNanResidual);
            P.x[r] = xn;
          }
          release(A, S, item++);
        }
      }
      if (!grid_barrier(A, S, bar_target)) return;
      mark(step, 5 * l + 4);
    }
    // -------------------------------------------------- LM
    {
      if (A.block_k > 0) {  // the last block's K-WTA, then output_norm
        bool a1, a2;
        mk_load_vec(P.x, P.d, S.xs, nullptr, 0.f, red, a1, a2);
        mk_block_kwta(S.xs, P.d, A.block_k, hist, nullptr);
        mk_norm_smem(S.xs, P.d, P.out_norm, P.eps, red, true, a2);
      } else {
        float v[kMkMaxVecPerThread];
#pragma unroll
        for (int k = 0; k < kMkMaxVecPerThread; ++k) {
          const int i = tid + k * kMkConsumers;
          v[k] = i < P.d ? __ldcg(P.x + i) : 0.f;
        }
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < kMkMaxVecPerThread; ++k) ss = fmaf(v[k], v[k], ss);
        ss = warp_sum(ss);
        if (lane == 0) red[wid] = ss;
        consumer_sync();
        float t = lane < kMkConsumerWarps ? red[lane] : 0.f;
        t = warp_sum(t);
        const float inv = 1.0f / sqrtf(t / (float)P.d + P.eps);
#pragma unroll
        for (int k = 0; k < kMkMaxVecPerThread; ++k) {
          const int i = tid + k * kMkConsumers;
          if (i < P.d) S.xs[i] = (v[k] * inv) * P.out_norm[i];
        }
        consumer_sync();
      }
      const float4* x4 = reinterpret_cast<const float4*>(S.xs);
      const int K4 = P.d >> 2;
      unsigned long long best = 0ull;
      const int rbeg = blockIdx.x * pl.lm_rows_per_cta;
      const int rend = min(P.V, rbeg + pl.lm_rows_per_cta);
      for (int r = rbeg; r < rend; r += pl.lm_stage_rows) {
        const int rows = min(pl.lm_stage_rows, rend - r);
        const unsigned char* slot = take(A, S, item);
        if (!slot) return;
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
          float s = warp_sum(a0 + a1);
          const int row = r + rr;
          if (P.lm_bias) s += P.lm_bias[row];
          if (lane == 0) P.logits[row] = s;
          const unsigned long long key = amax_key(s, (unsigned)row);
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
        }
      }
    }
    // the next step reads the new token and position
    if (!grid_barrier(A, S, bar_target)) return;
    mark(step, 5 * P.n_layers);
  }
}

__global__ void __launch_bounds__(kMkThreads, 1) k_decode_mega(MegaArgs A) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  MkShared S;
  S.full = reinterpret_cast<uint64_t*>(smem_raw);
  S.empty = S.full + kMkMaxSlots;
  S.abort_flag = reinterpret_cast<volatile int*>(S.empty + kMkMaxSlots);
  S.issued = S.abort_flag + 1;
  S.cabort = S.abort_flag + 2;
  S.xs = reinterpret_cast<float*>(smem_raw + kMkHeader);
  S.ps = S.xs + A.plan.xs_floats;
  S.part = S.ps + A.plan.ps_floats;
  S.slots = reinterpret_cast<unsigned char*>(S.part + kMkPartFloats);
  if (threadIdx.x == 0) {
    for (int i = 0; i < A.plan.nslots; ++i) {
      mbar_init(S.full + i, 1);
      mbar_init(S.empty + i, kMkConsumerWarps);
    }
    *S.abort_flag = 0;
    *S.issued = 0;
    *S.cabort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x >= kMkConsumers) {
    if (threadIdx.x == kMkConsumers) {
      mk_producer(A, S);
      // drain: every issued copy must land before the CTA may exit
      const int issued = *S.issued;
      for (int it = max(0, issued - A.plan.nslots); it < issued; ++it)
        mbar_wait(S.full + it % A.plan.nslots, (it / A.plan.nslots) & 1);
    }
    return;
  }
  mk_consumer(A, S);
}

}  // namespace gaje
