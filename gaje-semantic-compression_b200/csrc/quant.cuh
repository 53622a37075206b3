// quant.cuh -- the Q4_0 / Q8_0 quantisers on the device.
//
// quantize_q4_0_native (src/compute/quantize/python.rs:152-232) and the Q8_0
// arm beside it, as the host quantisers of flat_format.cpp compute them, for
// re-exporting large checkpoints without a round trip through host memory.
// Per 32 contiguous f32 values:
//   Q4_0: min, max (strict comparisons from +-f32::MAX, so NaN never wins);
//         scale = (max - min) / 15; inv = scale > 1e-7 ? 1 / scale : 0;
//         q = round_half_away((v - min) * inv) clamped to [0, 15] (NaN -> 0);
//         block {f16(scale), f16(min), qs[16]} with element 2k in the low
//         nibble of qs[k] (blocks.rs:9-31), f16 by round to nearest even.
//   Q8_0: max |v|; scale = max / 127; q = round_half_away(v * inv) clamped
//         to [-128, 127]; block {f16(scale), i8 qs[32]} (blocks.rs:37-50).
// Every operation is an explicit round-to-nearest intrinsic, so the bytes are
// the host quantisers' bytes (division included: __fdiv_rn is IEEE).
//
// Layout: a CTA quantises tiles of 256 blocks (32 KB of input).  The input
// tile is loaded with coalesced 16-byte loads into shared memory, float4
// slot c of block r stored at slot c ^ (r & 7), so that the 8 threads of a
// quarter-warp reading their own blocks' slot c touch 8 different slots; each
// thread quantises one block into a shared output tile, which is written back
// with coalesced 4-byte (Q4_0) or 2-byte (Q8_0) stores.  HBM-bound: 4 bytes
// read and 0.625 (Q4_0) or 1.0625 (Q8_0) bytes written per weight.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace gaje {

constexpr int kQuantThreads = 256;  // one block of 32 weights per thread per tile

// f32 -> f16 bits, round to nearest even, the half crate's conversion (the
// host twin is flat_format.cpp's f32_to_f16: NaN payloads quieted, >= 65520
// to infinity, subnormal results from |f| * 2^24 rounded to nearest even).
__device__ __forceinline__ uint16_t dev_f32_to_f16(float f) {
  const uint32_t x = __float_as_uint(f);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) {
    if (ax == 0x7F800000u) return uint16_t(sign | 0x7C00u);
    return uint16_t(sign | 0x7E00u | ((ax >> 13) & 0x3FFu));
  }
  if (ax >= 0x477FF000u) return uint16_t(sign | 0x7C00u);
  if (ax < 0x38800000u) {
    const float scaled = __fmul_rn(__uint_as_float(ax), 16777216.0f);  // exact power-of-two scaling
    return uint16_t(sign | uint32_t(rintf(scaled)));
  }
  const uint32_t t = ax - 0x38000000u + 0x0FFFu + ((ax >> 13) & 1u);
  return uint16_t(sign | (t >> 13));
}

__device__ __forceinline__ float rust_clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Loads tile `tile` (256 blocks, fewer at the end) into xs, swizzled.
__device__ __forceinline__ void quant_load_tile(const float4* w4, size_t nblocks, size_t tile, float4* xs) {
  const size_t b0 = tile * kQuantThreads;
  const size_t n4 = (nblocks - b0 < size_t(kQuantThreads) ? nblocks - b0 : size_t(kQuantThreads)) * 8;
  for (size_t i = threadIdx.x; i < n4; i += kQuantThreads) {
    const int r = int(i >> 3), c = int(i & 7);
    xs[r * 8 + (c ^ (r & 7))] = __ldcs(w4 + b0 * 8 + i);  // streamed once: evict first
  }
}

__global__ void __launch_bounds__(kQuantThreads) k_quantize_q4_0(const float* w, size_t nblocks, uint8_t* out) {
  __shared__ float4 xs[kQuantThreads * 8];
  __shared__ uint32_t os[kQuantThreads * 5];
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const size_t ntiles = (nblocks + kQuantThreads - 1) / kQuantThreads;
  for (size_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    quant_load_tile(w4, nblocks, tile, xs);
    __syncthreads();
    const size_t b0 = tile * kQuantThreads;
    const int nb = int(nblocks - b0 < size_t(kQuantThreads) ? nblocks - b0 : size_t(kQuantThreads));
    const int r = threadIdx.x;
    if (r < nb) {
      float v[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 f = xs[r * 8 + (c ^ (r & 7))];
        v[4 * c] = f.x;
        v[4 * c + 1] = f.y;
        v[4 * c + 2] = f.z;
        v[4 * c + 3] = f.w;
      }
      float mn = 3.40282347e+38f, mx = -3.40282347e+38f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (v[i] < mn) mn = v[i];
        if (v[i] > mx) mx = v[i];
      }
      const float scale = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
      const bool live = scale > 1e-7f;
      const float inv = live ? __fdiv_rn(1.0f, scale) : 0.0f;
      uint32_t word[5];
      word[0] = uint32_t(dev_f32_to_f16(scale)) | (uint32_t(dev_f32_to_f16(mn)) << 16);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t wd = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t q = 0;
          if (live) {
            const float rr = rust_clampf(roundf(__fmul_rn(__fsub_rn(v[8 * k + j], mn), inv)), 0.0f, 15.0f);
            q = (rr != rr) ? 0u : uint32_t(rr);
          }
          wd |= q << (4 * j);
        }
        word[1 + k] = wd;
      }
#pragma unroll
      for (int k = 0; k < 5; ++k) os[r * 5 + k] = word[k];
    }
    __syncthreads();
    uint32_t* o = reinterpret_cast<uint32_t*>(out + b0 * 20);
    for (int i = threadIdx.x; i < nb * 5; i += kQuantThreads) o[i] = os[i];
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kQuantThreads) k_quantize_q8_0(const float* w, size_t nblocks, uint8_t* out) {
  __shared__ float4 xs[kQuantThreads * 8];
  __shared__ uint16_t os[kQuantThreads * 17];
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const size_t ntiles = (nblocks + kQuantThreads - 1) / kQuantThreads;
  for (size_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    quant_load_tile(w4, nblocks, tile, xs);
    __syncthreads();
    const size_t b0 = tile * kQuantThreads;
    const int nb = int(nblocks - b0 < size_t(kQuantThreads) ? nblocks - b0 : size_t(kQuantThreads));
    const int r = threadIdx.x;
    if (r < nb) {
      float v[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 f = xs[r * 8 + (c ^ (r & 7))];
        v[4 * c] = f.x;
        v[4 * c + 1] = f.y;
        v[4 * c + 2] = f.z;
        v[4 * c + 3] = f.w;
      }
      float mx = 0.0f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float a = fabsf(v[i]);
        if (a > mx) mx = a;
      }
      const float scale = __fdiv_rn(mx, 127.0f);
      const bool live = scale > 1e-7f;
      const float inv = live ? __fdiv_rn(1.0f, scale) : 0.0f;
      os[r * 17] = dev_f32_to_f16(scale);
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        uint32_t pair = 0;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          int q = 0;
          if (live) {
            const float rr = rust_clampf(roundf(__fmul_rn(v[2 * k + j], inv)), -128.0f, 127.0f);
            q = (rr != rr) ? 0 : int(rr);
          }
          pair |= (uint32_t(q) & 0xFFu) << (8 * j);
        }
        os[r * 17 + 1 + k] = uint16_t(pair);
      }
    }
    __syncthreads();
    uint16_t* o = reinterpret_cast<uint16_t*>(out + b0 * 34);
    for (int i = threadIdx.x; i < nb * 17; i += kQuantThreads) o[i] = os[i];
    __syncthreads();
  }
}

}  // namespace gaje
