// tc_gemm.cuh -- Q4_0 matrix times many activation vectors on the 5th-gen
// tensor cores (tcgen05): the prefill and wide-batch projections, and the
// op-level M >= 16 path of gaje_cuda_q4_0_gemv (the isolated GEMM sweep at
// M = 64, 512).
//
// y[m][n] = flush(sum_k w_nk x_mk) + bias[n] with w = fma(q, scale, min) per
// element, the reference's own dequantisation (genomic.rs:267-336 AVX2 arm:
// dq = fma(q, scale, min), acc = fma(dq, x, acc)).  Both operands are split
// into bf16 pairs, v = hi + lo with hi = bf16(v) and lo = bf16(v - hi), and
// the product is taken as hi_w*hi_x + hi_w*lo_x + lo_w*hi_x (three
// kind::f16 MMAs into one f32 accumulator): the dropped lo*lo term and the
// split residues are below 3 * 2^-18 of each product, and accumulation is f32.
//
// Activations are split once per GEMM by k_tc_split (optionally fused with
// the RMSNorm that precedes the projection) into a tiled bf16 layout whose
// (32-K stage, 8-row group) blocks are the MMA's canonical K-major
// no-swizzle core-matrix layout: 8 rows x 16 bytes per core matrix, the
// four 8-element K chunks of a row group 128 B apart (LBO), row groups
// 512 B apart (SBO).  A CTA's activation tile for one stage is then one
// contiguous run per plane, fetched by a 1-D TMA bulk copy.
//
// CTA: 128 weight rows (the MMA's M) x NT vectors (its N), S stages of 32 K
// (one Q4 block per row; S = 4 at NT = 256, 4-6 for narrower tiles).
// Warp roles, each waiting only on the barriers it consumes:
// - warps 0-7 make the A tiles (two threads per weight row) and arrive on
//   a_full; for Q4 they dequantise raw words that lane 0 of warp 10 streams
//   from the K-block-major copy of the matrix through a shared-memory ring
//   with TMA bulk copies, tc_raw_stages(NT) stages ahead;
// - warp 8 lane 0 issues a stage's 2 k-steps x 3 MMAs once a_full and b_full
//   are complete and commits them to the stage's `done` barrier;
// - warp 9 lane 0 issues the activation copies of a stage (b_full, transaction
//   bytes) once `done` says the stage's previous MMAs are through.
// The epilogue reads the accumulator 32 columns per tcgen05.ld (one wait per
// 32 columns).
// The MMA lane never waits on an MMA completion, so the tensor pipe's queue
// stays full while the copies and the dequantisation run ahead.  The f32
// accumulator is NT columns of tensor memory; warp w < 8 reads lane quarter
// w%4, column half w/4, with tcgen05.ld for the epilogue.  With gridDim.z > 1
// the K stages are split across CTAs: partial tiles go to sp.part and
// k_tc_reduce adds them in split order and runs the epilogue.
#pragma once

#include <cuda_bf16.h>

#include "gemm.cuh"

namespace gaje {

constexpr int kTcProducers = 256;                 // warps 0-7: two threads per weight row
constexpr int kTcMmaWarp = kTcProducers / 32;     // lane 0 issues the MMAs
constexpr int kTcCopyWarp = kTcMmaWarp + 1;       // lane 0 issues the activation copies
constexpr int kTcLoadWarp = kTcMmaWarp + 2;       // streams raw Q4 words (Q4 sources)
constexpr int kTcThreads = kTcProducers + 96;
constexpr int kTcRows = 128;                      // weight rows per CTA (MMA M)
constexpr int kTcK = 32;                          // K per stage: one Q4 block of every row
constexpr int kTcChunks = kTcK / 8;               // 16-byte K chunks of a row per stage
constexpr unsigned kTcKidTimeout = 15;

__host__ __device__ constexpr size_t tc_stage_bytes(int nt) {
  return size_t(2) * kTcRows * kTcK * 2 + size_t(2) * nt * kTcK * 2;  // A hi/lo + B hi/lo (bf16)
}
// Raw Q4 words of one stage (128 rows x 16 B nibbles + 128 x 4 B scale/min),
// tc_raw_stages(NT) of them in flight ahead of the dequantising warps.  A
// narrow tile has little MMA work per stage, so its weight stream must run
// further ahead to cover the HBM latency: 8 slots (20 KB) at 256 vectors,
// 40 (100 KB) at 16-32.
constexpr int kTcRawSlot = kTcRows * 20;
__host__ __device__ constexpr int tc_raw_stages(int nt) { return nt >= 256 ? 8 : nt >= 128 ? 24 : nt >= 64 ? 32 : 40; }
// MMA stages: as many as fit beside the raw ring in 213 KB, at most 8 (four
// at 256 vectors, a stage is 48 KB there; six at 16 vectors, 18 KB).
__host__ __device__ constexpr int tc_stages(int nt) {
  return int((213 * 1024 - 1024 - tc_raw_stages(nt) * kTcRawSlot) / tc_stage_bytes(nt)) > 8
             ? 8
             : int((213 * 1024 - 1024 - tc_raw_stages(nt) * kTcRawSlot) / tc_stage_bytes(nt));
}
__host__ __device__ constexpr size_t tc_smem_bytes(int nt) {  // 1 KB header (barriers, TMEM address)
  return 1024 + size_t(tc_stages(nt)) * tc_stage_bytes(nt) + size_t(tc_raw_stages(nt)) * kTcRawSlot;
}
static_assert(3 * 8 + 2 * 40 <= 126, "the barriers and the TMEM address fit the 1 KB header");
__host__ __device__ constexpr int tc_tmem_cols(int nt) { return nt < 32 ? 32 : nt; }
// Bytes of one bf16 plane of split activations for Mpad rows x K.
__host__ __device__ inline size_t tc_plane_bytes(int mpad, int K) { return size_t(mpad) * K * 2; }

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
// 32 lanes x N consecutive 32-bit columns of tensor memory into N registers
// per thread (one load, one wait).
template <int N>
__device__ __forceinline__ void tc_ld(uint32_t taddr, float (&v)[N]);
template <>
__device__ __forceinline__ void tc_ld<8>(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tc_ld<16>(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tc_ld<32>(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
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

// Byte offset of (row r, 8-element K chunk c) in a K-major no-swizzle stage
// tile with 32 K per row: core matrix (r/8, c) at (r/8)*512 + c*128 (LBO 128
// between K chunks, SBO 512 between row groups), row r%8 at +16.
constexpr uint32_t kTcLbo = 128, kTcSbo = kTcChunks * 128;
__device__ __forceinline__ uint32_t tc_off(int r, int c) {
  return uint32_t((r >> 3) * kTcSbo + c * kTcLbo + (r & 7) * 16);
}
// Byte offset of (row r, K chunk c) in the split-activation planes of mpad rows:
// stage c/4, row group r/8, chunk c%4, row r%8 -- a CTA's activation tile of
// one stage is one contiguous run.
__host__ __device__ __forceinline__ size_t tc_xoff(int r, int c, int mpad) {
  return ((size_t(c / kTcChunks) * (mpad >> 3) + (r >> 3)) * kTcChunks + (c % kTcChunks)) * 128 + (r & 7) * 16;
}

// Weight sources of the A operand.  Q4Rows (kRawRing): the loader lane
// copies each stage's raw words (one Q4 block of each of the 128 rows) from
// the K-block-major copy of the matrix -- qsT[kb][row], smT[kb][row], rows
// ld apart, so a stage is one contiguous run of each -- into a shared-memory
// ring tc_raw_stages(NT) deep with two 1-D TMA bulk copies, tracked by an
// mbarrier; warps 0-7 dequantise them into the A tiles, two threads per row
// (half a block each).  The converters issue no global
// loads, so the proxy fence that publishes their tile writes to the tensor
// cores waits on nothing else.  F32Rows: a thread owns 16 consecutive
// elements (half h of a 32-element block) of one row per stage, kDepth
// stages ahead in registers.
struct Q4Rows {  // Q4_0: w = fma(q, scale, min) (genomic.rs:267-336)
  Q4View W;
  const uint4* qsT;     // [nb][ld] 16-byte nibble words, K-block major
  const uint32_t* smT;  // [nb][ld] scale | min << 16
  int ld;               // rows of a K block in qsT / smT: N rounded up to a multiple of 4
  static constexpr bool kRawRing = true;  // words staged through shared memory by the loader lane
  struct Regs {
    uint2 q;
    uint32_t s;
  };
  __host__ __device__ __forceinline__ int N() const { return W.N; }
  __host__ __device__ __forceinline__ int K() const { return W.K; }
  __host__ __device__ __forceinline__ const float* bias() const { return W.bias; }
  // rows [row0, row0 + 128) of block blk into a raw slot: slot rows past ld
  // keep whatever they held (their outputs are dropped); both runs start on
  // 16-byte boundaries and are multiples of 16 bytes (ld % 4 == 0)
  __device__ __forceinline__ void issue_raw(unsigned char* slot, int row0, int blk, uint64_t* bar) const {
    const int rows = min(kTcRows, ld - row0);
    const size_t o = (size_t)blk * ld + row0;
    mbar_expect_tx(bar, uint32_t(rows) * 20u);
    const uint64_t pol = l2_policy_evict_first();  // read once per step: keep L2 for the activations
    bulk_g2s_hint(slot, qsT + o, uint32_t(rows) * 16u, bar, pol);
    bulk_g2s_hint(slot + kTcRows * 16, smT + o, uint32_t(rows) * 4u, bar, pol);
  }
  // half h (16 elements) of slot row rl
  __device__ __forceinline__ void read_raw(Regs& g, const unsigned char* slot, int rl, int h) const {
    g.q = *reinterpret_cast<const uint2*>(slot + rl * 16 + h * 8);
    g.s = *reinterpret_cast<const uint32_t*>(slot + kTcRows * 16 + rl * 4);
  }
  __device__ __forceinline__ void values(const Regs& g, int w, float (&v)[8]) const {
    float sc, mn;
    unpack_sm(g.s, sc, mn);
    const uint32_t wd = w == 0 ? g.q.x : g.q.y;
#pragma unroll
    for (int e = 0; e < 8; ++e)  // exact q: the nibble in the mantissa of 2^23, minus 2^23
      v[e] = fmaf(__uint_as_float(((wd >> (4 * e)) & 0xFu) | 0x4B000000u) - 8388608.0f, sc, mn);
  }
};
struct F32Rows {  // plain f32 rows [N][K] (the lm_head, linear/forward.rs:20-32)
  const float* W;
  const float* b;
  int n, k;
  static constexpr bool kRawRing = false;
  static constexpr int kDepth = 4;  // stages of rows in flight per thread (a register ring)
  struct Regs {
    float4 f[4];
  };
  __host__ __device__ __forceinline__ int N() const { return n; }
  __host__ __device__ __forceinline__ int K() const { return k; }
  __host__ __device__ __forceinline__ const float* bias() const { return b; }
  __device__ __forceinline__ void load(Regs& g, int r, int blk, int h) const {
    const float4* p = reinterpret_cast<const float4*>(W + (size_t)r * k + blk * 32 + h * 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) g.f[i] = __ldcs(p + i);
  }
  __device__ __forceinline__ void zero(Regs& g) const {
#pragma unroll
    for (int i = 0; i < 4; ++i) g.f[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __device__ __forceinline__ void values(const Regs& g, int w, float (&v)[8]) const {
    const float4 a = g.f[2 * w], c = g.f[2 * w + 1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
  }
};

// x [M][K] f32 (optionally RMSNorm'd: (x * inv) * w, norm.rs:17-87) -> the
// split planes hi/lo [mpad rows]; rows M..mpad-1 are zero.  One CTA of
// kTsThreads per row (the sum of squares by a block reduction, added warp by
// warp in a fixed order); launch mpad CTAs.  With st, the block-input and
// normed-output NaN guards (block/forward.rs:11-13, :22-24) at pos[row].
struct TcSplitArgs {
  const float* x;
  int M, K, mpad;
  const float* norm_w;  // nullptr: no norm
  float eps;
  unsigned char* hi;
  unsigned char* lo;
  DevState* st;
  const unsigned* pos;
  int layer;
};
constexpr int kTsThreads = 256;
__global__ void __launch_bounds__(kTsThreads) k_tc_split(TcSplitArgs A) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[kTsThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int r = blockIdx.x;
  if (r >= A.mpad) return;
  const bool live = r < A.M;
  const float* xr = A.x + (size_t)(live ? r : 0) * A.K;
  float inv = 1.f;
  const bool norm = A.norm_w && live;  // uniform over the CTA
  if (norm) {
    float ss = 0.f;
    int bad = 0;
    for (int j = tid; j < (A.K >> 2); j += kTsThreads) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(xr) + j);
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
      bad |= (v.x != v.x) | (v.y != v.y) | (v.z != v.z) | (v.w != v.w);
    }
    ss = warp_sum(ss);
    if (lane == 0) red[wid] = ss;
    bad = __syncthreads_or(bad);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kTsThreads / 32; ++w) tot += red[w];
    inv = 1.0f / sqrtf(tot / (float)A.K + A.eps);
    if (A.st && bad && tid == 0) nan_flag(A.st, A.pos[r], A.layer, kNanInput);
  }
  int bad_out = 0;
  for (int c = tid; c < (A.K >> 3); c += kTsThreads) {
    float v[8];
    if (live) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(xr + c * 8));
      const float4 b = __ldg(reinterpret_cast<const float4*>(xr + c * 8) + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      if (A.norm_w) {
        const float4 wa = __ldg(reinterpret_cast<const float4*>(A.norm_w + c * 8));
        const float4 wb = __ldg(reinterpret_cast<const float4*>(A.norm_w + c * 8) + 1);
        const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          v[i] = (v[i] * inv) * w[i];
          bad_out |= (v[i] != v[i]);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    uint4 hi, lo;
    tc_split8(v, hi, lo);
    const size_t off = tc_xoff(r, c, A.mpad);
    *reinterpret_cast<uint4*>(A.hi + off) = hi;
    *reinterpret_cast<uint4*>(A.lo + off) = lo;
  }
  if (A.st && norm) {
    bad_out = __syncthreads_or(bad_out);
    if (bad_out && tid == 0) nan_flag(A.st, A.pos[r], A.layer, kNanAttnNorm);
  }
}

// Split-K work area: part[z][M][N] f32 partial tiles, finished by k_tc_reduce.
struct TcSplit {
  float* part = nullptr;
};

// Launch: grid (ceil(N/128), mpad/NT, Z), kTcThreads, tc_smem_bytes(NT);
// K % 64 == 0; the K stages are divided evenly over Z (Z > 1 needs sp).
template <int NT, class WS, class Epi>
__global__ void __launch_bounds__(kTcThreads, 1) k_q4_gemm_tc(WS W, const unsigned char* xhi,
                                                           const unsigned char* xlo, int M, int mpad, TcSplit sp,
                                                           Epi epi, DevState* st) {
  static_assert(NT % 16 == 0 && NT >= 16 && NT <= 256, "MMA N");
  constexpr int S = tc_stages(NT);
  extern __shared__ __align__(1024) unsigned char tc_smem[];
  uint64_t* a_full = reinterpret_cast<uint64_t*>(tc_smem);  // [S] 128 producer arrivals
  uint64_t* b_full = a_full + S;                             // [S] activation copies landed
  uint64_t* done = b_full + S;                               // [S] MMAs of the stage complete
  constexpr int R = tc_raw_stages(NT);
  uint64_t* raw_full = done + S;                             // [R] raw words landed
  uint64_t* raw_empty = raw_full + R;                        // [R] raw words read
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tc_smem + 1016);
  unsigned char* stage0 = tc_smem + 1024;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int row0 = blockIdx.x * kTcRows, m0 = blockIdx.y * NT;
  const int nkt = W.K() / kTcK;
  const int Z = gridDim.z;
  const int kb = (nkt * (int)blockIdx.z) / Z, ke = (nkt * ((int)blockIdx.z + 1)) / Z;
  const int n = ke - kb;  // stages of this CTA
  constexpr uint32_t kA = kTcRows * kTcK * 2, kB = NT * kTcK * 2;  // bytes of one bf16 plane
  constexpr int kCols = tc_tmem_cols(NT);
  if (wid == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(uint32_t(kCols)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(a_full + s, kTcProducers);
      mbar_init(b_full + s, 1);
      mbar_init(done + s, 1);
    }
    for (int s = 0; s < R; ++s) {
      mbar_init(raw_full + s, 1);              // the loader lane's arrival with the copies' bytes
      mbar_init(raw_empty + s, kTcProducers);  // one per converter thread
    }
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  int issued = 0, committed = -1;  // the issue lane's copies and last commit (for the drain)
  if (wid < kTcProducers / 32) {
    if constexpr (WS::kRawRing) {
      // ---------------- converters: rows (t & 7) | ((t >> 4) << 3), half (t >> 3) & 1 -- the
      // eight threads of a quarter warp write eight consecutive 16-byte rows of a core matrix
      unsigned char* raw0 = stage0 + S * tc_stage_bytes(NT);
      const int rl = (tid & 7) | ((tid >> 4) << 3), h = (tid >> 3) & 1;
      pdl_wait();
      pdl_trigger();
      for (int i = 0; i < n; ++i) {
        const int s = i % S, slot = i % R;
        if (i >= S && !(ok = mbar_wait(done + s, ((i / S) - 1) & 1))) break;  // the stage's previous MMAs
        if (!(ok = mbar_wait(raw_full + slot, (i / R) & 1))) break;
        typename WS::Regs g;
        W.read_raw(g, raw0 + slot * kTcRawSlot, rl, h);
        unsigned char* A_hi = stage0 + s * tc_stage_bytes(NT);
        unsigned char* A_lo = A_hi + kA;
#pragma unroll
        for (int w = 0; w < 2; ++w) {  // chunk w of the thread's 16 elements = stage chunk 2h + w
          float v[8];
          W.values(g, w, v);
          uint4 hi, lo;
          tc_split8(v, hi, lo);
          const uint32_t off = tc_off(rl, 2 * h + w);
          *reinterpret_cast<uint4*>(A_hi + off) = hi;
          *reinterpret_cast<uint4*>(A_lo + off) = lo;
        }
        // the slot is released only once its words have been used: the next TMA
        // copy into it (asynchronous proxy) must not overtake a read still in flight
        mbar_arrive(raw_empty + slot);
        fence_async_smem();  // these generic-proxy writes, visible to the tensor cores
        mbar_arrive(a_full + s);
      }
    } else {
      // ---------------- f32 rows: thread t = weight row row0 + t/2, half t&1 of the stage's block
      const int rl = tid >> 1, h = tid & 1;
      const int r = row0 + rl;
      const bool rok = r < W.N();
      constexpr int P = WS::kDepth;
      typename WS::Regs g[P];
      #pragma unroll
      for (int u = 0; u < P; ++u) {  // weights never depend on the previous kernel
        W.zero(g[u]);
        if (rok && u < n) W.load(g[u], r, kb + u, h);
      }
      pdl_wait();
      pdl_trigger();
      #pragma unroll 1
      for (int i0 = 0; i0 < n; i0 += P) {
        #pragma unroll
        for (int u = 0; u < P; ++u) {  // stage i's words sit in ring entry i % P
          const int i = i0 + u;
          if (i < n) {
            const int s = i % S;
            unsigned char* A_hi = stage0 + s * tc_stage_bytes(NT);
            unsigned char* A_lo = A_hi + kA;
            if (i >= S && ok) ok = mbar_wait(done + s, ((i / S) - 1) & 1);  // the stage's previous MMAs are done
            const typename WS::Regs gc = g[u];
            if (i + P < n && rok) W.load(g[u], r, kb + i + P, h);  // P stages ahead
            #pragma unroll
            for (int w = 0; w < 2; ++w) {  // chunk w of the thread's 16 elements = stage chunk 2h + w
              float v[8];
              W.values(gc, w, v);
              uint4 hi, lo;
              tc_split8(v, hi, lo);
              const uint32_t off = tc_off(rl, 2 * h + w);
              *reinterpret_cast<uint4*>(A_hi + off) = hi;
              *reinterpret_cast<uint4*>(A_lo + off) = lo;
            }
            fence_async_smem();  // these generic-proxy writes, visible to the tensor cores
            mbar_arrive(a_full + s);
          }
        }
      }
    }
  } else if (wid == kTcLoadWarp) {
    // ---------------- loader lane (Q4): each stage's block of the 128 rows, up to
    // R stages ahead; weights never depend on the previous kernel
    if constexpr (WS::kRawRing) {
      if (lane == 0) {
        unsigned char* raw0 = stage0 + S * tc_stage_bytes(NT);
        int j = 0;
        for (; j < n; ++j) {
          const int slot = j % R;
          if (j >= R && !(ok = mbar_wait(raw_empty + slot, ((j / R) - 1) & 1))) break;
          W.issue_raw(raw0 + slot * kTcRawSlot, row0, kb + j, raw_full + slot);
        }
        // none of these copies may still land in shared memory when the CTA
        // exits: wait (bounded) for the latest copy of every slot used
        for (int t = j - 1; t >= 0 && t >= j - R; --t) mbar_wait(raw_full + t % R, (t / R) & 1);
      }
    }
    pdl_wait();
    pdl_trigger();
  } else if (wid == kTcMmaWarp) {
    // ---------------- MMA warp: a stage's MMAs as soon as its A and B tiles are in
    pdl_wait();
    pdl_trigger();
    if (lane == 0) {
      constexpr uint32_t idesc = tc_idesc(kTcRows, NT);
      for (int i = 0; i < n; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!(ok = mbar_wait(b_full + s, ph) && mbar_wait(a_full + s, ph))) break;
        tc_fence_after();
        unsigned char* A_hi = stage0 + s * tc_stage_bytes(NT);
        const uint32_t ah = smem_u32(A_hi), al = ah + kA, bh = al + kA, bl = bh + kB;
#pragma unroll
        for (int k = 0; k < kTcK / 16; ++k) {  // a 16-wide k-step spans two core matrices: +256 B
          const uint32_t o = uint32_t(k) * 2u * kTcLbo;
          const uint64_t dah = tc_desc(ah + o, kTcLbo, kTcSbo), dal = tc_desc(al + o, kTcLbo, kTcSbo);
          const uint64_t dbh = tc_desc(bh + o, kTcLbo, kTcSbo), dbl = tc_desc(bl + o, kTcLbo, kTcSbo);
          tc_mma(tmem, dah, dbh, idesc, (i > 0 || k > 0) ? 1u : 0u);
          tc_mma(tmem, dah, dbl, idesc, 1u);
          tc_mma(tmem, dal, dbh, idesc, 1u);
        }
        tc_commit(done + s);
        committed = i;
      }
    }
  } else {
    // ---------------- copy warp: a stage's activation tiles as soon as its previous MMAs are through
    pdl_wait();
    pdl_trigger();
    if (lane == 0) {
      const size_t gstride = tc_plane_bytes(mpad, kTcK);  // bytes of one stage of a plane
      for (int j = 0; j < n; ++j) {
        const int s = j % S;
        if (j >= S && !(ok = mbar_wait(done + s, ((j / S) - 1) & 1))) break;
        unsigned char* B_hi = stage0 + s * tc_stage_bytes(NT) + 2 * kA;
        const size_t src = size_t(kb + j) * gstride + size_t(m0 >> 3) * kTcSbo;
        mbar_expect_tx(b_full + s, 2 * kB);
        bulk_g2s(B_hi, xhi + src, kB, b_full + s);
        bulk_g2s(B_hi + kB, xlo + src, kB, b_full + s);
        issued = j + 1;
      }
    }
  }
  // the last commit covers every MMA issued before it
  constexpr int kIssueWarp = kTcMmaWarp;
  if (wid < kIssueWarp && n > 0) {
    const bool fin = mbar_wait(done + (n - 1) % S, ((n - 1) / S) & 1);
    ok = ok && fin;
  }
  ok = __syncthreads_and(ok) != 0;
  if (!ok) {
    if (tid == 0 && st) flag_timeout(st, kTcKidTimeout);
    // nothing may still write shared or tensor memory when they are released:
    // wait (bounded again) for the last MMAs and every stage's latest copy
    if (wid == kTcMmaWarp && lane == 0 && committed >= 0) mbar_wait(done + committed % S, (committed / S) & 1);
    if (wid == kTcCopyWarp && lane == 0) {
      for (int s = 0; s < S && s < issued; ++s) {
        const int j = s + S * ((issued - 1 - s) / S);  // the stage's latest copy
        mbar_wait(b_full + s, (j / S) & 1);
      }
    }
  }
  tc_fence_after();
  if (ok && wid < kIssueWarp) {
    // warp w reads TMEM lanes 32*(w%4).. (its quarter), columns of half w/4
    const int q = wid & 3;
    const int rr = row0 + q * 32 + lane;  // TMEM lane = tile row
    const int WN = W.N();
    const bool has0 = rr < WN;
    const float* bp = W.bias();
    const float bias = (bp && has0) ? __ldg(bp + rr) : 0.f;  // this lane's row
    constexpr int kHalf = NT / 2 < 8 ? 8 : NT / 2;
    constexpr int kC = kHalf < 32 ? kHalf : 32;  // columns per TMEM load (kHalf is a multiple)
    const int cb = (wid >> 2) * kHalf, ce = min(NT, cb + kHalf);
#pragma unroll 1
    for (int c0 = cb; c0 < ce; c0 += kC) {
      float v[kC];
      tc_ld<kC>(tmem + (uint32_t(q * 32) << 16) + uint32_t(c0), v);
      if (Z > 1) {  // partial tile -> part[z][m][row]
#pragma unroll
        for (int j = 0; j < kC; ++j)
          if (has0 && m0 + c0 + j < M) sp.part[((size_t)blockIdx.z * M + m0 + c0 + j) * WN + rr] = v[j];
      } else {
        // row pair (r0, r0 + 1) = lanes (2p, 2p + 1): of columns j, j + 1 the even lane
        // finishes column j and the odd lane column j + 1, one exchange per column pair
        const bool odd = lane & 1;
        const int r0 = rr & ~1;
        const bool p0 = r0 < WN, p1 = r0 + 1 < WN;
#pragma unroll
        for (int j = 0; j < kC; j += 2) {
          const float fa = flush_small(v[j]) + bias, fb = flush_small(v[j + 1]) + bias;
          const float recv = __shfl_xor_sync(0xffffffffu, odd ? fa : fb, 1);
          const int col = m0 + c0 + j + (odd ? 1 : 0);
          if (p0 && col < M) epi(col, r0, odd ? recv : fa, p1, odd ? fb : recv);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (wid == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(uint32_t(kCols)));
}

// The split-K finish: y = flush(sum_z part[z][m][row]) + bias through epi,
// the splits added in order.  One thread per (vector, row pair); launch
// ceil(M * ceil(N/2) / 256) CTAs of 256 threads.
template <class Epi>
__global__ void __launch_bounds__(256) k_tc_reduce(const float* part, int Z, int M, int N, const float* bias,
                                                   Epi epi) {
  pdl_wait();
  pdl_trigger();
  const int np = (N + 1) >> 1;
  const long it = (long)blockIdx.x * 256 + threadIdx.x;
  if (it >= (long)M * np) return;
  const int m = int(it / np), r0 = 2 * int(it - (long)m * np);
  const bool has1 = r0 + 1 < N;
  float s0 = 0.f, s1 = 0.f;
  if ((N & 1) == 0) {  // row pairs are 8-byte aligned: eight splits' loads in flight, added in split order
    const size_t zs = (size_t)M * N;
    const float* p = part + (size_t)m * N + r0;
#pragma unroll 1
    for (int z0 = 0; z0 < Z; z0 += 8) {
      float2 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        v[u] = z0 + u < Z ? __ldcg(reinterpret_cast<const float2*>(p + (z0 + u) * zs)) : make_float2(0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (z0 + u < Z) {
          s0 += v[u].x;
          s1 += v[u].y;
        }
    }
  } else {
    for (int z = 0; z < Z; ++z) {
      const float* p = part + ((size_t)z * M + m) * N + r0;
      s0 += __ldcg(p);
      if (has1) s1 += __ldcg(p + 1);
    }
  }
  const float b0 = bias ? __ldg(bias + r0) : 0.f;
  const float b1 = (bias && has1) ? __ldg(bias + r0 + 1) : 0.f;
  epi(m, r0, flush_small(s0) + b0, has1, flush_small(s1) + b1);
}

}  // namespace gaje
