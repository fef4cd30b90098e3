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

// Counts every kernel launch this library queues (tb_launch_count): called right after each
// launch, whether it went through launch() or a <<<>>> of its own.
void note_launch();

// ---- launches with programmatic dependent launch -------------------------------------------
// The memory-bound kernels are launched with programmatic dependent launch (PDL) allowed: the
// GPU may schedule a kernel's CTAs while the previous kernel of the stream is still draining,
// so the launch latency (about 0.8 us between back-to-back launches on B200, 0.2-0.6 us less
// with PDL) overlaps that kernel's tail. Such a kernel starts with pdl_wait()
// (griddepcontrol.wait: returns once the previous kernel has completed and its memory is
// visible) before it touches global memory, then pdl_release() (griddepcontrol.launch_dependents)
// lets the next PDL kernel be scheduled; the next kernel waits for this one's completion all
// the same. Without the launch attribute both instructions do nothing. TESTT_B200_PDL=0 in the
// environment launches without the attribute (plain stream ordering).

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

bool pdl_enabled();

// Launches `kernel` (whose first statements are pdl_wait(); pdl_release();) on `stream`;
// TB_OK or TB_ELAUNCH with the CUDA message.
template <typename... KArgs, typename... Args>
int launch(const char *what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
           cudaStream_t stream, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return set_error(TB_ELAUNCH, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  note_launch();
  return TB_OK;
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

// ---- bulk async copies and mbarriers (sm_90+ PTX, used on sm_100a) -------------------------
// 1-D bulk copy global -> shared completing on an mbarrier (no multicast). Every wait on an
// mbarrier is bounded: after kWaitLimit polls the waiter gives up, counts a timeout in
// g_wait_timeouts (read by tb_wait_timeouts) and the kernel returns instead of hanging.

constexpr uint32_t kWaitLimit = 1u << 24;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// true once the phase with the given parity has completed; false after `limit` polls
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity,
                                          uint32_t limit = kWaitLimit) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// Bounded waits that gave up, on the current device since the library was loaded. One counter
// per translation unit (no relocatable device code); a file whose kernels wait registers a
// reader with TB_REGISTER_TIMEOUT_READER and tb_wait_timeouts sums them.
static __device__ unsigned int g_wait_timeouts = 0;

typedef cudaError_t (*TimeoutReader)(unsigned int *);
int register_timeout_reader(TimeoutReader reader);

#define TB_REGISTER_TIMEOUT_READER(tag)                                             \
  static cudaError_t tag##_read_timeouts(unsigned int *out) {                       \
    return cudaMemcpyFromSymbol(out, ::tb::g_wait_timeouts, sizeof(unsigned int));  \
  }                                                                                 \
  static const int tag##_timeout_reader = ::tb::register_timeout_reader(tag##_read_timeouts);

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
