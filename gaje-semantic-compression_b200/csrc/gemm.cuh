// gemm.cuh -- Q4_0 matrix times a few activation vectors (the op-level M > 1
// path of gaje_cuda_q4_0_gemv, SURVEY configs[2] M = 8).
//
// y[m][n] = flush(sum_b scale_b*A_b + min_b*X_b) + bias[n] with
// A_b = sum_k q_k x_mk over block b (the AVX2 arm of genomic.rs:267-336
// factored, as in the decode kernels).  Every weight block is read and turned
// into nibble values once per CTA and applied to MT activation vectors held in
// shared memory (swizzled, pre-scaled per nibble slot, with per-block sums), K
// staged in chunks so that any K fits.  A warp owns a row pair for the whole
// K range (the pair shares its activation loads), lanes over the blocks of a
// chunk, a shuffle reduction at the end.
#pragma once

#include "megakernel.cuh"

namespace gaje {

constexpr int kSkThreads = 256;
constexpr int kSkWarps = kSkThreads / 32;
constexpr int kSkChunk = 1024;  // activations per vector per staged chunk (32 blocks)

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

// epi(m, r0, v0, has1, v1) receives rows r0 (and r0 + 1) of vector m, flushed
// and with the bias added.
template <int MT, class Epi>
__global__ void __launch_bounds__(kSkThreads) k_q4_gemm_skinny(Q4View W, const float* x, int M, Epi epi) {
  extern __shared__ __align__(16) float sk_smem[];
  float* xs = sk_smem;                    // [MT][kSkChunk]
  float* xsum = sk_smem + MT * kSkChunk;  // [MT][kSkChunk / 32]
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int m0 = blockIdx.y * MT;
  const int mt = min(MT, M - m0);
  const int r0 = (blockIdx.x * kSkWarps + wid) * 2;
  const bool has0 = r0 < W.N, has1 = r0 + 1 < W.N;
  float acc0[MT], acc1[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    acc0[m] = 0.f;
    acc1[m] = 0.f;
  }
  const uint4* q0p = W.qs + (size_t)min(r0, W.N - 1) * W.nb;
  const uint4* q1p = W.qs + (size_t)min(r0 + 1, W.N - 1) * W.nb;
  const uint32_t* s0p = W.sm + (size_t)min(r0, W.N - 1) * W.nbp;
  const uint32_t* s1p = W.sm + (size_t)min(r0 + 1, W.N - 1) * W.nbp;
  for (int k0 = 0; k0 < W.K; k0 += kSkChunk) {
    const int kc = min(kSkChunk, W.K - k0);  // a multiple of 32
    __syncthreads();                          // the previous chunk is consumed
    for (int m = 0; m < MT; ++m) {
      for (int i = tid; i < kc; i += kSkThreads) {  // whole warps per 32-block (kc % 32 == 0)
        const float v = m < mt ? __ldg(x + (size_t)(m0 + m) * W.K + k0 + i) : 0.f;
        xs[m * kSkChunk + swz(i)] = v * nib_prescale(i & 7);
        const float bs = warp_sum(v);
        if (lane == 0) xsum[m * (kSkChunk / 32) + (i >> 5)] = bs;
      }
    }
    __syncthreads();
    if (has0) {
      const int nbc = kc >> 5, b0 = k0 >> 5;
      for (int bl = lane; bl < nbc; bl += 32) {
        const int b = b0 + bl;
        const uint4 qa = __ldg(q0p + b);
        const uint4 qb = has1 ? __ldg(q1p + b) : make_uint4(0u, 0u, 0u, 0u);
        float sc0, mn0, sc1, mn1;
        unpack_sm(__ldg(s0p + b), sc0, mn0);
        unpack_sm(has1 ? __ldg(s1p + b) : 0u, sc1, mn1);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          float A0, A1;
          q4_pair_qx(qa, qb, has1, xs + m * kSkChunk, bl, A0, A1);
          const float xb = xsum[m * (kSkChunk / 32) + bl];
          acc0[m] = fmaf(sc0, A0, fmaf(mn0, xb, acc0[m]));
          acc1[m] = fmaf(sc1, A1, fmaf(mn1, xb, acc1[m]));
        }
      }
    }
  }
  if (!has0) return;
  const float b0 = W.bias ? __ldg(W.bias + r0) : 0.f;
  const float b1 = (W.bias && has1) ? __ldg(W.bias + r0 + 1) : 0.f;
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const float v0 = warp_sum(acc0[m]), v1 = warp_sum(acc1[m]);
    if (lane == 0 && m < mt) epi(m0 + m, r0, flush_small(v0) + b0, has1, flush_small(v1) + b1);
  }
}

}  // namespace gaje
