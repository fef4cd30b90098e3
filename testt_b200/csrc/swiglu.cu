// Gated SiLU (SwiGLU) forward and in-place backward for sm_100a.
//
// Reference: solution/mlp.py:31-40 (gated_silu_fwd_kernel), :43-58
// (gated_silu_bwd_inplace_kernel), launches :61-77. Flat grid-stride over 8-value vectors of the
// [rows, inter] output: each vector is one 16-byte load of gate, one of up (and of dact in
// backward) and one or two 16-byte stores, fully coalesced. The math is the reference's formula in
// fp32 with the fast exponential and division the reference's tl.exp / fp32 divide also lower to
// (__expf, __fdividef); the result is rounded once to fp16.
#include "common.cuh"

namespace tb {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 2;

__device__ __forceinline__ float silu(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

__device__ __forceinline__ void swiglu_bwd_one(float dact, float g, float u, float &dg, float &du) {
  const float sig = __fdividef(1.0f, 1.0f + __expf(-g));
  const float d_silu = dact * u;
  dg = d_silu * sig * (1.0f + g * (1.0f - sig));
  du = dact * (g * sig);
}

// Vector index i (8 values) -> (row, chunk) with one invariant division; n < 2^32 vectors.
__global__ void __launch_bounds__(kThreads)
    swiglu_fwd_vec(const uint16_t *__restrict__ gu, uint16_t *__restrict__ act, uint32_t n,
                   FastDiv vpr, int64_t inter) {
  const uint32_t stride = gridDim.x * kThreads;
  for (uint32_t i0 = blockIdx.x * kThreads * kUnroll + threadIdx.x; i0 < n;
       i0 += stride * kUnroll) {
    float g[kUnroll][8], u[kUnroll][8];
#pragma unroll
    for (int r = 0; r < kUnroll; ++r) {
      const uint32_t i = i0 + r * kThreads;
      if (i < n) {
        uint32_t row, c;
        vpr.divmod(i, row, c);
        const uint16_t *p = gu + (int64_t)row * 2 * inter + c * 8;
        load8h(p, g[r]);
        load8h(p + inter, u[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < kUnroll; ++r) {
      const uint32_t i = i0 + r * kThreads;
      if (i < n) {
        uint32_t row, c;
        vpr.divmod(i, row, c);
        float o[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = silu(g[r][k]) * u[r][k];
        store8h(act + (int64_t)row * inter + c * 8, o);
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads)
    swiglu_bwd_vec(const uint16_t *__restrict__ dact, uint16_t *__restrict__ gu, uint32_t n,
                   FastDiv vpr, int64_t inter) {
  const uint32_t stride = gridDim.x * kThreads;
  for (uint32_t i0 = blockIdx.x * kThreads * kUnroll + threadIdx.x; i0 < n;
       i0 += stride * kUnroll) {
    float d[kUnroll][8], g[kUnroll][8], u[kUnroll][8];
#pragma unroll
    for (int r = 0; r < kUnroll; ++r) {
      const uint32_t i = i0 + r * kThreads;
      if (i < n) {
        uint32_t row, c;
        vpr.divmod(i, row, c);
        uint16_t *p = gu + (int64_t)row * 2 * inter + c * 8;
        load8h(dact + (int64_t)row * inter + c * 8, d[r]);
        load8h_rw(p, g[r]);
        load8h_rw(p + inter, u[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < kUnroll; ++r) {
      const uint32_t i = i0 + r * kThreads;
      if (i < n) {
        uint32_t row, c;
        vpr.divmod(i, row, c);
        uint16_t *p = gu + (int64_t)row * 2 * inter + c * 8;
        float dg[8], du[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) swiglu_bwd_one(d[r][k], g[r][k], u[r][k], dg[k], du[k]);
        store8h(p, dg);
        store8h(p + inter, du);
      }
    }
  }
}

__device__ __forceinline__ float f16(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t h16(float f) { return __half_as_ushort(__float2half_rn(f)); }

__global__ void swiglu_fwd_any(const uint16_t *gu, uint16_t *act, int64_t rows, int64_t inter) {
  const int64_t n = rows * inter;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / inter, c = i - row * inter;
    const float g = f16(gu[row * 2 * inter + c]), u = f16(gu[row * 2 * inter + inter + c]);
    act[i] = h16(silu(g) * u);
  }
}

__global__ void swiglu_bwd_any(const uint16_t *dact, uint16_t *gu, int64_t rows, int64_t inter) {
  const int64_t n = rows * inter;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / inter, c = i - row * inter;
    uint16_t *p = gu + row * 2 * inter + c;
    float dg, du;
    swiglu_bwd_one(f16(dact[i]), f16(p[0]), f16(p[inter]), dg, du);
    p[0] = h16(dg);
    p[inter] = h16(du);
  }
}

unsigned blocks_for(int64_t n, int per_block) {
  int64_t b = (n + per_block - 1) / per_block;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (b > cap) b = cap;
  return (unsigned)(b > 0 ? b : 1);
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" int tb_swiglu_fwd(const uint16_t *gu, uint16_t *act, int64_t rows, int64_t inter,
                             void *stream) {
  if (rows < 0 || inter <= 0)
    return set_error(TB_EINVAL, "swiglu_fwd: rows %lld inter %lld", (long long)rows, (long long)inter);
  if (rows == 0) return TB_OK;
  if (!gu || !act) return set_error(TB_EINVAL, "swiglu_fwd: gu and act are required");
  cudaStream_t st = as_stream(stream);
  const int64_t nvec = rows * (inter / 8);
  if (inter % 8 == 0 && nvec < (1LL << 31) && aligned(gu, 16) && aligned(act, 16)) {
    swiglu_fwd_vec<<<blocks_for(nvec, kThreads * kUnroll), kThreads, 0, st>>>(
        gu, act, (uint32_t)nvec, FastDiv((uint32_t)(inter / 8)), inter);
  } else {
    swiglu_fwd_any<<<blocks_for(rows * inter, kThreads), kThreads, 0, st>>>(gu, act, rows, inter);
  }
  return check_launch("swiglu_fwd");
}

extern "C" int tb_swiglu_bwd_inplace(const uint16_t *dact, uint16_t *gu, int64_t rows,
                                     int64_t inter, void *stream) {
  if (rows < 0 || inter <= 0)
    return set_error(TB_EINVAL, "swiglu_bwd: rows %lld inter %lld", (long long)rows, (long long)inter);
  if (rows == 0) return TB_OK;
  if (!gu || !dact) return set_error(TB_EINVAL, "swiglu_bwd: dact and gu are required");
  cudaStream_t st = as_stream(stream);
  const int64_t nvec = rows * (inter / 8);
  if (inter % 8 == 0 && nvec < (1LL << 31) && aligned(gu, 16) && aligned(dact, 16)) {
    swiglu_bwd_vec<<<blocks_for(nvec, kThreads * kUnroll), kThreads, 0, st>>>(
        dact, gu, (uint32_t)nvec, FastDiv((uint32_t)(inter / 8)), inter);
  } else {
    swiglu_bwd_any<<<blocks_for(rows * inter, kThreads), kThreads, 0, st>>>(dact, gu, rows, inter);
  }
  return check_launch("swiglu_bwd");
}
