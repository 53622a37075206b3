// tc_gemm.cuh -- Q4_0 matrix times many activation vectors on the 5th-gen
// tensor cores (tcgen05): the prefill and wide-batch projections, and the
// op-level M >= 16 path of gaje_cuda_q4_0_gemv (SURVEY configs[2] M = 64,
// 512).
//
// y[m][n] = flush(sum_k w_nk x_mk) + bias[n] with w = fma(q, scale, min) per
// element, the reference's own dequantisation (genomic.rs:267-336 AVX2 arm:
// dq = fma(q, scale, min), acc = fma(dq, x, acc)).  Both operands are split
// into bf16 pairs, v = hi + lo with hi = bf16(v) and lo = bf16(v - hi), and
// the product is taken as hi_w*hi_x + hi_w*lo_x + lo_w*hi_x (three
// kind::f16 MMAs into one f32 accumulator): the dropped lo*lo term and the
// split residues are ~2^-16 of each product, so the sums keep about 16
// significant bits per product and full f32 accumulation.
//
// CTA tile: 128 weight rows (the MMA's M) x NT vectors (its N), K in stages
// of 64 (two Q4 blocks), two stages in shared memory.  All 128 threads
// produce a stage -- thread t dequantises row t's two blocks, and the threads
// together split the NT x 64 activation tile -- into the K-major
// no-swizzle canonical layout (8-row x 16-byte core matrices, LBO = 128 B
// between the two K halves of a core-matrix pair, SBO = 1024 B between
// 8-row groups); thread 0 issues 4 k-steps x 3 MMAs per stage and commits
// them to the stage's mbarrier, which the producers wait on before
// overwriting that stage two stages later.  The f32 accumulator lives in
// tensor memory (NT columns x 128 lanes); the epilogue reads it with
// tcgen05.ld (warp w: lanes 32w..32w+31 = its 32 rows).
#pragma once

#include <cuda_bf16.h>

#include "gemm.cuh"

namespace gaje {

constexpr int kTcThreads = 128;
constexpr int kTcRows = 128;     // weight rows per CTA (MMA M)
constexpr int kTcK = 64;         // K per stage
constexpr int kTcStages = 2;
constexpr unsigned kTcKidTimeout = 15;

__host__ __device__ constexpr size_t tc_stage_bytes(int nt) {
  return size_t(2) * kTcRows * kTcK * 2 + size_t(2) * nt * kTcK * 2;  // A hi/lo + B hi/lo (bf16)
}
__host__ __device__ constexpr size_t tc_smem_bytes(int nt) {
  return 1024 + kTcStages * tc_stage_bytes(nt);  // 1 KB header (barriers, TMEM address) + stages
}
__host__ __device__ constexpr int tc_tmem_cols(int nt) { return nt < 32 ? 32 : nt; }

// Shared-memory matrix descriptor, K-major, no swizzle (version 1 for sm_100):
// start >> 4 in [0,14), LBO >> 4 in [16,30), SBO >> 4 in [32,46), bit 46 set.
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}
// Instruction descriptor of kind::f16: f32 accumulator (bit 4), bf16 A and B
// (bits 7, 10), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t tc_idesc(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// 32 lanes x 8 consecutive 32-bit columns of tensor memory into 8 registers.
__device__ __forceinline__ void tc_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// (hi, lo) bf16 pairs of 8 consecutive floats: 16 bytes each.
__device__ __forceinline__ void tc_split8(const float (&v)[8], uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 bh = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    const float2 fh = __bfloat1622float2(bh);
    const __nv_bfloat162 bl = __floats2bfloat162_rn(v[2 * i] - fh.x, v[2 * i + 1] - fh.y);
    h[i] = *reinterpret_cast<const uint32_t*>(&bh);
    l[i] = *reinterpret_cast<const uint32_t*>(&bl);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Byte offset of (row r, 8-element K chunk c) in a K-major no-swizzle tile
// with 64 K per row: core matrix (r/8, c) at (r/8)*1024 + c*128, row r%8 at +16.
__device__ __forceinline__ uint32_t tc_off(int r, int c) { return uint32_t((r >> 3) * 1024 + c * 128 + (r & 7) * 16); }

// Launch: grid (ceil(N/128), ceil(M/NT)), kTcThreads, tc_smem_bytes(NT);
// K % 64 == 0; x rows 16-byte aligned.  `st` receives a timeout code.
template <int NT, class Epi>
__global__ void __launch_bounds__(kTcThreads) k_q4_gemm_tc(Q4View W, const float* x, int M, Epi epi, DevState* st) {
  static_assert(NT % 16 == 0 && NT >= 16 && NT <= 256, "MMA N");
  extern __shared__ __align__(1024) unsigned char tc_smem[];
  uint64_t* done = reinterpret_cast<uint64_t*>(tc_smem);        // [kTcStages] MMA-complete barriers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tc_smem + 64);
  unsigned char* stage0 = tc_smem + 1024;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int row0 = blockIdx.x * kTcRows, m0 = blockIdx.y * NT;
  const int nk = W.K / kTcK;
  constexpr uint32_t kA = kTcRows * kTcK * 2, kB = NT * kTcK * 2;  // bytes of one bf16 plane
  constexpr int kCols = tc_tmem_cols(NT);
  if (wid == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(uint32_t(kCols)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int s = 0; s < kTcStages; ++s) mbar_init(done + s, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_trigger();
  const int r = row0 + tid;  // this thread's weight row
  const bool rok = r < W.N;
  const uint4* qrow = W.qs + (size_t)min(r, W.N - 1) * W.nb;
  const uint32_t* srow = W.sm + (size_t)min(r, W.N - 1) * W.nbp;
  constexpr uint32_t idesc = tc_idesc(kTcRows, NT);
  bool ok = true;
  for (int kt = 0; kt < nk; ++kt) {
    const int s = kt & 1;
    unsigned char* A_hi = stage0 + s * tc_stage_bytes(NT);
    unsigned char* A_lo = A_hi + kA;
    unsigned char* B_hi = A_lo + kA;
    unsigned char* B_lo = B_hi + kB;
    if (kt >= kTcStages && ok) ok = mbar_wait(done + s, ((kt - kTcStages) >> 1) & 1);  // MMAs of kt-2 done
    // A: row r, blocks 2kt and 2kt+1 -> w = fma(q, scale, min) -> (hi, lo)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int b = 2 * kt + h;
      uint4 q = make_uint4(0u, 0u, 0u, 0u);
      uint32_t smv = 0u;
      if (rok) {
        q = __ldg(qrow + b);
        smv = __ldg(srow + b);
      }
      float sc, mn;
      unpack_sm(smv, sc, mn);
      const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {  // word w = elements 8w..8w+7 of the block = chunk 4h + w
        float v[8];
#pragma unroll
        for (int n = 0; n < 8; ++n) v[n] = fmaf(float((wd[w] >> (4 * n)) & 0xFu), sc, mn);
        uint4 hi, lo;
        tc_split8(v, hi, lo);
        const uint32_t off = tc_off(tid, 4 * h + w);
        *reinterpret_cast<uint4*>(A_hi + off) = hi;
        *reinterpret_cast<uint4*>(A_lo + off) = lo;
      }
    }
    // B: NT vectors x 8 chunks of 8 floats
    for (int it = tid; it < NT * 8; it += kTcThreads) {
      const int vr = it >> 3, c = it & 7;
      float v[8];
      if (m0 + vr < M) {
        const float4* src = reinterpret_cast<const float4*>(x + (size_t)(m0 + vr) * W.K + kt * kTcK + c * 8);
        const float4 a = __ldg(src), bq = __ldg(src + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = bq.x; v[5] = bq.y; v[6] = bq.z; v[7] = bq.w;
      } else {
#pragma unroll
        for (int n = 0; n < 8; ++n) v[n] = 0.f;
      }
      uint4 hi, lo;
      tc_split8(v, hi, lo);
      const uint32_t off = tc_off(vr, c);
      *reinterpret_cast<uint4*>(B_hi + off) = hi;
      *reinterpret_cast<uint4*>(B_lo + off) = lo;
    }
    fence_async_smem();  // the generic-proxy writes above, visible to the tensor cores
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && ok) {
      tc_fence_after();
      const uint32_t ah = smem_u32(A_hi), al = smem_u32(A_lo), bh = smem_u32(B_hi), bl = smem_u32(B_lo);
#pragma unroll
      for (int k = 0; k < kTcK / 16; ++k) {  // a 16-wide k-step spans two core matrices: +256 B
        const uint32_t o = uint32_t(k) * 256u;
        const uint64_t dah = tc_desc(ah + o, 128, 1024), dal = tc_desc(al + o, 128, 1024);
        const uint64_t dbh = tc_desc(bh + o, 128, 1024), dbl = tc_desc(bl + o, 128, 1024);
        tc_mma(tmem, dah, dbh, idesc, (kt > 0 || k > 0) ? 1u : 0u);
        tc_mma(tmem, dah, dbl, idesc, 1u);
        tc_mma(tmem, dal, dbh, idesc, 1u);
      }
      tc_commit(done + s);
    }
  }
  // the last commit covers every MMA issued before it
  if (ok && nk > 0) ok = mbar_wait(done + ((nk - 1) & 1), ((nk - 1) >> 1) & 1);
  if (!ok) {
    if (tid == 0 && st) flag_timeout(st, kTcKidTimeout);
    // let any MMA still in flight finish before the tensor memory is freed (bounded again)
    if (nk > 0) mbar_wait(done + ((nk - 1) & 1), ((nk - 1) >> 1) & 1);
  }
  tc_fence_after();
  if (ok) {
    const int rr = row0 + wid * 32 + lane;  // TMEM lane = tile row
    const bool has0 = rr < W.N;
    const float bias = (W.bias && has0) ? __ldg(W.bias + rr) : 0.f;
    const float bias1 = __shfl_down_sync(0xffffffffu, bias, 1);
    const bool has1 = rr + 1 < W.N;
#pragma unroll 1
    for (int c0 = 0; c0 < NT; c0 += 8) {
      float v[8];
      tc_ld8(tmem + (uint32_t(wid * 32) << 16) + uint32_t(c0), v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float f = flush_small(v[j]);
        const float f1 = __shfl_down_sync(0xffffffffu, f, 1);  // row rr + 1
        if ((lane & 1) == 0 && has0 && m0 + c0 + j < M) epi(m0 + c0 + j, rr, f + bias, has1, f1 + bias1);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (wid == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(uint32_t(kCols)));
}

}  // namespace gaje
