// sample.cuh -- nucleus (top-p) sampling on the device.
//
// sample_top_p_core (src/compute/sampling.rs:14-55): p_i = exp((l_i - max) /
// T), normalised; tokens sorted by descending p (a stable sort: equal p keep
// index order); the nucleus is the shortest prefix whose running sum exceeds
// top_p; the token is the first of the nucleus whose running sum reaches
// r * (the nucleus' sum).  The reference draws r from thread_rng; here the
// caller passes it (a seeded stream makes runs reproducible).
//
// One CTA of 1024 threads, no sort and no scratch memory: the order "p
// descending, then index ascending" is walked by radix selection on the bit
// pattern of p (non-negative floats order as their bits), 8 bits per pass,
// with a per-bucket count and probability mass.  Masses are 2^-40 fixed point
// in 64-bit integers: integer atomics give the same sums in any order, so the
// choice is deterministic (the reference's f32 running sums differ from these
// exact ones by rounding, which matters only for an r or a top_p within a
// rounding of a boundary).  The probabilities are recomputed from the logits
// in every pass (cheap next to the passes' bandwidth).  Two selections:
//   1. the key v1 at which the descending running mass first exceeds
//      top_p * total, and how many of the tokens with p == v1 (in index order)
//      the nucleus takes;
//   2. within the nucleus, the key v2 at which the running mass first reaches
//      r * (nucleus mass); the token is the j-th with p == v2 in index order.
#pragma once

#include <stdint.h>

namespace gaje {

constexpr int kSampleThreads = 1024;
constexpr double kSampleFix = 1099511627776.0;  // 2^40

struct TopPShared {
  unsigned long long mass[256];
  unsigned cnt[256];
  unsigned long long scan[kSampleThreads / 32];
  unsigned key, found, j;
  unsigned long long above, above_cnt;
  float mx;
  unsigned out;
};

__device__ __forceinline__ float tp_prob(const float* lg, int i, float mx, float temperature) {
  const float p = expf(__fdiv_rn(__fsub_rn(lg[i], mx), temperature));
  return p == p ? p : 0.0f;
}
__device__ __forceinline__ unsigned long long tp_fixed(float p) {
  return (unsigned long long)__double2ull_rn(double(p) * kSampleFix);
}

// Radix selection over the tokens with key > limit (all with limit = -1 as
// unsigned... use has_limit): the largest key v whose inclusion makes the
// running mass (descending keys) cross target: strict -> mass > target, else
// mass >= target.  Leaves in S: key, above (mass of eligible keys > v),
// above_cnt (their count), found, and cnt of v in S.j.  Not found: above is
// the eligible total.
__device__ void tp_select(const float* lg, int n, float temperature, bool has_limit, unsigned limit, double target,
                          bool strict, TopPShared& S) {
  const int tid = threadIdx.x;
  const int chunk = (n + kSampleThreads - 1) / kSampleThreads;
  const int lo = min(n, tid * chunk), hi = min(n, lo + chunk);
  unsigned prefix = 0, mask = 0;
  if (tid == 0) {
    S.above = 0;
    S.above_cnt = 0;
    S.found = 1;
  }
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < 256; b += kSampleThreads) {
      S.mass[b] = 0ull;
      S.cnt[b] = 0u;
    }
    __syncthreads();
    const float mx = S.mx;
    for (int i = lo; i < hi; ++i) {
      const float p = tp_prob(lg, i, mx, temperature);
      const unsigned key = __float_as_uint(p);
      if (has_limit && key <= limit) continue;
      if ((key & mask) != prefix) continue;
      const unsigned b = (key >> shift) & 0xFFu;
      atomicAdd(&S.cnt[b], 1u);
      atomicAdd(&S.mass[b], tp_fixed(p));
    }
    __syncthreads();
    if (tid == 0 && S.found) {
      unsigned long long acc = S.above, acc_cnt = S.above_cnt;
      int hit = -1;
      for (int b = 255; b >= 0; --b) {
        if (!S.cnt[b]) continue;
        const double tot = double(acc + S.mass[b]);
        if (strict ? tot > target : tot >= target) {
          hit = b;
          break;
        }
        acc += S.mass[b];
        acc_cnt += S.cnt[b];
      }
      S.above = acc;
      S.above_cnt = acc_cnt;
      if (hit < 0) {
        S.found = 0;
      } else {
        S.key = (prefix | (unsigned(hit) << shift));
        S.j = S.cnt[hit];
      }
    }
    __syncthreads();
    if (!S.found) return;
    prefix = S.key;
    mask |= 0xFFu << shift;
  }
}

// The index of the j-th (1-based) token with key == v, in index order.
__device__ void tp_nth_equal(const float* lg, int n, float temperature, unsigned v, unsigned j, TopPShared& S) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int chunk = (n + kSampleThreads - 1) / kSampleThreads;
  const int lo = min(n, tid * chunk), hi = min(n, lo + chunk);
  const float mx = S.mx;
  unsigned c = 0;
  for (int i = lo; i < hi; ++i) c += __float_as_uint(tp_prob(lg, i, mx, temperature)) == v;
  // exclusive prefix of the per-thread counts (thread order = index order)
  unsigned incl = c;
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) S.scan[wid] = incl;
  __syncthreads();
  if (tid == 0) {
    unsigned long long run = 0;
    for (int w = 0; w < kSampleThreads / 32; ++w) {
      const unsigned long long t = S.scan[w];
      S.scan[w] = run;
      run += t;
    }
  }
  __syncthreads();
  const unsigned before = unsigned(S.scan[wid]) + incl - c;
  if (c && j > before && j <= before + c) {
    unsigned k = before;
    for (int i = lo; i < hi; ++i)
      if (__float_as_uint(tp_prob(lg, i, mx, temperature)) == v && ++k == j) {
        S.out = unsigned(i);
        break;
      }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kSampleThreads) k_sample_top_p(const float* lg, int n, float temperature, float top_p,
                                                                 float r, unsigned* out, unsigned* kept) {
  __shared__ TopPShared S;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  __shared__ float redm[kSampleThreads / 32];
  float m = -INFINITY;
  for (int i = tid; i < n; i += kSampleThreads) m = fmaxf(m, lg[i]);
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) redm[wid] = m;
  __syncthreads();
  if (tid == 0) {
    float b = -INFINITY;
    for (int w = 0; w < kSampleThreads / 32; ++w) b = fmaxf(b, redm[w]);
    S.mx = b;
    S.out = 0u;
  }
  __syncthreads();
  // total mass (every token)
  tp_select(lg, n, temperature, false, 0u, 1e300, true, S);  // never crosses: S.above = total
  const unsigned long long total = S.above;
  const unsigned long long n_all = S.above_cnt;
  if (total == 0ull) {  // sum_exp <= 0 (sampling.rs:24-26)
    if (tid == 0) {
      *out = 0u;
      if (kept) *kept = 0u;
    }
    return;
  }
  // 1. the nucleus
  tp_select(lg, n, temperature, false, 0u, double(top_p) * double(total), true, S);
  const bool all = !S.found;
  unsigned v1 = 0, j1 = 0;
  unsigned long long above1 = 0, kept_mass = total, kept_cnt = n_all;
  if (!all) {
    v1 = S.key;
    above1 = S.above;
    const unsigned long long f1 = tp_fixed(__uint_as_float(v1));
    const double need = double(top_p) * double(total) - double(above1);  // > above1 + (j-1) f1, <= above1 + j f1
    j1 = f1 ? unsigned(min(double(S.j), floor(need / double(f1)) + 1.0)) : S.j;
    j1 = max(1u, j1);
    kept_mass = above1 + (unsigned long long)j1 * f1;
    kept_cnt = S.above_cnt + j1;
  }
  // 2. the token: first of the nucleus whose running mass reaches r * kept
  const double t2 = double(r) * double(kept_mass);
  unsigned v2, j2;
  if (!all && t2 > double(above1)) {  // among the nucleus' tokens with p == v1
    const unsigned long long f1 = tp_fixed(__uint_as_float(v1));
    v2 = v1;
    j2 = f1 ? unsigned(ceil((t2 - double(above1)) / double(f1))) : 1u;
    j2 = min(max(1u, j2), j1);
  } else {
    tp_select(lg, n, temperature, !all, v1, t2, false, S);
    if (!S.found) {  // rounding: the first token of the order (sampling.rs:54)
      tp_select(lg, n, temperature, false, 0u, 0.0, false, S);
    }
    v2 = S.key;
    const unsigned long long f2 = tp_fixed(__uint_as_float(v2));
    j2 = f2 ? unsigned(ceil((t2 - double(S.above)) / double(f2))) : 1u;
    j2 = min(max(1u, j2), S.j);
  }
  tp_nth_equal(lg, n, temperature, v2, j2, S);
  if (tid == 0) {
    *out = S.out;
    if (kept) *kept = unsigned(kept_cnt);
  }
}

}  // namespace gaje
