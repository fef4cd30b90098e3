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

__device__ __forceinline__ float silu(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

__device__ __forceinline__ void swiglu_bwd_one(float dact, float g, float u, float &dg, float &du) {
  const float sig = __fdividef(1.0f, 1.0f + __expf(-g));
  const float d_silu = dact * u;
  dg = d_silu * sig * (1.0f + g * (1.0f - sig));
  du = dact * (g * sig);
}

__device__ __forceinline__ void unpack8(const uint4 &v, float (&f)[8]) {
  const float2 a = unpack_half2(v.x), b = unpack_half2(v.y), c = unpack_half2(v.z),
               d = unpack_half2(v.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

// Vector index i (8 values) -> (row, chunk) with one invariant division; n < 2^32 vectors.
// Grid-stride with the next vector's 16-byte loads issued before the current vector's math
// (one vector in flight ahead per thread, raw in registers). The forward is launched with a
// grid that covers every vector (one per thread, the most loads in flight at the start), the
// backward with one wave of resident blocks (measured fastest for each at 621 and 2048 rows).
__global__ void __launch_bounds__(kThreads)
    swiglu_fwd_vec(const uint16_t *__restrict__ gu, uint16_t *__restrict__ act, uint32_t n,
                   FastDiv vpr, int64_t inter) {
  pdl_wait();
  pdl_release();
  const uint32_t stride = gridDim.x * kThreads;
  uint32_t i = blockIdx.x * kThreads + threadIdx.x;
  if (i >= n) return;
  uint32_t row, c;
  vpr.divmod(i, row, c);
  const uint16_t *p = gu + (int64_t)row * 2 * inter + c * 8;
  uint4 gb = __ldg(reinterpret_cast<const uint4 *>(p));
  uint4 ub = __ldg(reinterpret_cast<const uint4 *>(p + inter));
  while (true) {
    float g[8], u[8], o[8];
    unpack8(gb, g);
    unpack8(ub, u);
    const uint32_t r0 = row, c0 = c;
    const uint32_t next = i + stride;
    const bool more = next < n && next > i;
    if (more) {
      vpr.divmod(next, row, c);
      p = gu + (int64_t)row * 2 * inter + c * 8;
      gb = __ldg(reinterpret_cast<const uint4 *>(p));
      ub = __ldg(reinterpret_cast<const uint4 *>(p + inter));
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = silu(g[k]) * u[k];
    store8h(act + (int64_t)r0 * inter + c0 * 8, o);
    if (!more) break;
    i = next;
  }
}

__global__ void __launch_bounds__(kThreads)
    swiglu_bwd_vec(const uint16_t *__restrict__ dact, uint16_t *__restrict__ gu, uint32_t n,
                   FastDiv vpr, int64_t inter) {
  pdl_wait();
  pdl_release();
  const uint32_t stride = gridDim.x * kThreads;
  uint32_t i = blockIdx.x * kThreads + threadIdx.x;
  if (i >= n) return;
  uint32_t row, c;
  vpr.divmod(i, row, c);
  uint16_t *p = gu + (int64_t)row * 2 * inter + c * 8;
  uint4 db = __ldg(reinterpret_cast<const uint4 *>(dact + (int64_t)row * inter + c * 8));
  uint4 gb = *reinterpret_cast<const uint4 *>(p);
  uint4 ub = *reinterpret_cast<const uint4 *>(p + inter);
  while (true) {
    float d[8], g[8], u[8], dg[8], du[8];
    unpack8(db, d);
    unpack8(gb, g);
    unpack8(ub, u);
    uint16_t *const out = p;
    const uint32_t next = i + stride;
    const bool more = next < n && next > i;
    if (more) {
      vpr.divmod(next, row, c);
      p = gu + (int64_t)row * 2 * inter + c * 8;
      db = __ldg(reinterpret_cast<const uint4 *>(dact + (int64_t)row * inter + c * 8));
      gb = *reinterpret_cast<const uint4 *>(p);
      ub = *reinterpret_cast<const uint4 *>(p + inter);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) swiglu_bwd_one(d[k], g[k], u[k], dg[k], du[k]);
    store8h(out, dg);
    store8h(out + inter, du);
    if (!more) break;
    i = next;
  }
}

__device__ __forceinline__ float f16(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t h16(float f) { return __half_as_ushort(__float2half_rn(f)); }

__global__ void swiglu_fwd_any(const uint16_t *gu, uint16_t *act, int64_t rows, int64_t inter) {
  pdl_wait();
  pdl_release();
  const int64_t n = rows * inter;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / inter, c = i - row * inter;
    const float g = f16(gu[row * 2 * inter + c]), u = f16(gu[row * 2 * inter + inter + c]);
    act[i] = h16(silu(g) * u);
  }
}

__global__ void swiglu_bwd_any(const uint16_t *dact, uint16_t *gu, int64_t rows, int64_t inter) {
  pdl_wait();
  pdl_release();
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

// Blocks of kThreads for n work items, at most `cap` (a grid-stride loop covers the rest).
unsigned blocks_for(int64_t n, int64_t cap) {
  int64_t b = (n + kThreads - 1) / kThreads;
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
    return launch("swiglu_fwd", swiglu_fwd_vec, blocks_for(nvec, 1LL << 24), kThreads, 0, st, gu,
                  act, (uint32_t)nvec, FastDiv((uint32_t)(inter / 8)), inter);
  }
  return launch("swiglu_fwd", swiglu_fwd_any, blocks_for(rows * inter, (int64_t)sm_count() * 16),
                kThreads, 0, st, gu, act, rows, inter);
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
    static const int wave = resident_blocks(swiglu_bwd_vec, kThreads);
    return launch("swiglu_bwd", swiglu_bwd_vec, blocks_for(nvec, wave), kThreads, 0, st, dact, gu,
                  (uint32_t)nvec, FastDiv((uint32_t)(inter / 8)), inter);
  }
  return launch("swiglu_bwd", swiglu_bwd_any, blocks_for(rows * inter, (int64_t)sm_count() * 16),
                kThreads, 0, st, dact, gu, rows, inter);
}
