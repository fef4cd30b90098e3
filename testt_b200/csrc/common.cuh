// Shared helpers of the testt_b200 kernels: error reporting of the C ABI, fp16 packing,
// block reductions. Everything here is sm_100a device code or plain host C++.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/testt_b200.h"
#include "fastdiv.h"

namespace tb {

// ---- error reporting (one message per host thread) -----------------------------------------

int set_error(int code, const char *fmt, ...);

// Checks the launch just queued; returns TB_OK or TB_ELAUNCH with the CUDA message.
int check_launch(const char *what);

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void *p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// Number of SMs of the current device (cached per device).
int sm_count();

// Blocks of `kernel` resident on the whole device at `threads` threads and `smem` dynamic shared
// bytes per block (the occupancy calculator times the SM count; at least the SM count).
template <typename Kernel>
int resident_blocks(Kernel kernel, int threads, size_t smem = 0) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  return per_sm * sm_count();
}

// ---- fp16 packing --------------------------------------------------------------------------

// Two floats rounded to nearest-even fp16 and packed (one cvt.rn.f16x2.f32).
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ float2 unpack_half2(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2 *>(&v);
  return __half22float2(h);
}

// 8 fp16 values in a 16-byte vector <-> 8 floats.
__device__ __forceinline__ void load8h(const uint16_t *p, float (&f)[8]) {
  uint4 v = __ldg(reinterpret_cast<const uint4 *>(p));
  float2 a = unpack_half2(v.x), b = unpack_half2(v.y), c = unpack_half2(v.z),
         d = unpack_half2(v.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

// Same, without the read-only path (for buffers the kernel also writes).
__device__ __forceinline__ void load8h_rw(const uint16_t *p, float (&f)[8]) {
  uint4 v = *reinterpret_cast<const uint4 *>(p);
  float2 a = unpack_half2(v.x), b = unpack_half2(v.y), c = unpack_half2(v.z),
         d = unpack_half2(v.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

__device__ __forceinline__ void store8h(uint16_t *p, const float (&f)[8]) {
  uint4 v;
  v.x = pack_half2(f[0], f[1]);
  v.y = pack_half2(f[2], f[3]);
  v.z = pack_half2(f[4], f[5]);
  v.w = pack_half2(f[6], f[7]);
  *reinterpret_cast<uint4 *>(p) = v;
}

__device__ __forceinline__ void load8f(const float *p, float (&f)[8]) {
  float4 a = __ldg(reinterpret_cast<const float4 *>(p));
  float4 b = __ldg(reinterpret_cast<const float4 *>(p + 4));
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

__device__ __forceinline__ void store8f(float *p, const float (&f)[8]) {
  reinterpret_cast<float4 *>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4 *>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}

// Streaming (evict-first) 16-byte store for outputs that are not re-read by this kernel.
__device__ __forceinline__ void store8h_cs(uint16_t *p, const float (&f)[8]) {
  uint4 v;
  v.x = pack_half2(f[0], f[1]);
  v.y = pack_half2(f[2], f[3]);
  v.z = pack_half2(f[4], f[5]);
  v.w = pack_half2(f[6], f[7]);
  __stcs(reinterpret_cast<uint4 *>(p), v);
}

// ---- reductions ----------------------------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over the block; `scratch` holds >= 32 floats. Every thread gets the total.
__device__ __forceinline__ float block_sum(float v, float *scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();  // scratch may still be read by a previous call
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = lane < nwarps ? scratch[lane] : 0.f;
  return warp_sum(t);
}

}  // namespace tb
