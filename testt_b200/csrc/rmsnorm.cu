// Residual add + RMSNorm, forward and backward, for sm_100a.
//
// Reference: solution/rmsnorm.py:24-43 (rmsnorm_fwd_kernel), :46-69 (rmsnorm_bwd_kernel) and
// their launches :76-112. One CTA per token row, as in the reference, but the row lives in
// registers: each thread owns NCH chunks of 8 consecutive values, read and written with 16-byte
// (fp16) or 2x16-byte (fp32) vector accesses, and the row sum is a warp-shuffle + shared-memory
// reduction. For hidden = 1536 that is 192 threads with one chunk each: one pass over HBM for
// every tensor, nothing re-read.
//
// Operation order follows the reference: s = x + delta; rstd = 1 / sqrt(sum(s^2) / H + eps)
// (IEEE sqrt and division); y = (s * rstd) * w. Backward: g = (dy + dypad) * w; n = s * rstd;
// dx = (g - n * sum(g n) / H) * rstd + ds.
#include "common.cuh"

namespace tb {
namespace {

template <int NCH>
__global__ void rmsnorm_fwd_vec(const float *__restrict__ x, const uint16_t *__restrict__ delta,
                                const float *__restrict__ w, float *__restrict__ s_out,
                                uint16_t *__restrict__ y, float *__restrict__ ypad,
                                const int64_t *__restrict__ pad_idx, float *__restrict__ rstd_out,
                                int64_t hidden, float eps) {
  pdl_wait();
  pdl_release();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nch = (int)(hidden / 8);
  const int64_t base = row * hidden;
  // every load of the row is issued before the reduction: x, delta, weight and the pad row
  const int64_t dest = ypad != nullptr ? __ldg(pad_idx + row) * hidden : 0;
  float v[NCH][8], wv[NCH][8];
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nch) {
      load8f(x + base + c * 8, v[i]);
      load8f(w + c * 8, wv[i]);
      if (delta != nullptr) {
        float d[8];
        load8h(delta + base + c * 8, d);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[i][k] = v[i][k] + d[k];
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nch) {
      if (delta != nullptr) store8f(s_out + base + c * 8, v[i]);
#pragma unroll
      for (int k = 0; k < 8; ++k) ss += v[i][k] * v[i][k];
    }
  }
  const float total = block_sum(ss, red);
  const float rstd = 1.0f / sqrtf(total / (float)hidden + eps);
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nch) {
      float o[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = __fmul_rn(__fmul_rn(v[i][k], rstd), wv[i][k]);
      store8h(y + base + c * 8, o);
      if (ypad != nullptr) store8f(ypad + dest + c * 8, o);
    }
  }
  if (threadIdx.x == 0) rstd_out[row] = rstd;
}

template <int NCH>
__global__ void rmsnorm_bwd_vec(const float *__restrict__ s, const float *__restrict__ rstd_in,
                                const float *__restrict__ w, const uint16_t *__restrict__ dy,
                                const float *__restrict__ dypad,
                                const int64_t *__restrict__ pad_idx, const float *__restrict__ ds,
                                float *__restrict__ dx, uint16_t *__restrict__ ddelta,
                                int64_t hidden) {
  pdl_wait();
  pdl_release();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nch = (int)(hidden / 8);
  const int64_t base = row * hidden;
  const int64_t src = dypad != nullptr ? __ldg(pad_idx + row) * hidden : 0;
  const float rstd = __ldg(rstd_in + row);
  // g, n and the residual gradient are all loaded before the reduction
  float g[NCH][8], n[NCH][8], r[NCH][8];
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nch) {
      float wv[8];
      if (dy != nullptr) {
        load8h(dy + base + c * 8, g[i]);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) g[i][k] = 0.f;
      }
      if (dypad != nullptr) {
        float p[8];
        load8f(dypad + src + c * 8, p);
#pragma unroll
        for (int k = 0; k < 8; ++k) g[i][k] = g[i][k] + p[k];
      }
      if (ds != nullptr) {
        load8f(ds + base + c * 8, r[i]);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) r[i][k] = 0.f;
      }
      load8f(w + c * 8, wv);
      load8f(s + base + c * 8, n[i]);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        g[i][k] = g[i][k] * wv[k];
        n[i][k] = n[i][k] * rstd;
        dot += g[i][k] * n[i][k];
      }
    }
  }
  const float proj = block_sum(dot, red) / (float)hidden;
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nch) {
      float o[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        o[k] = (g[i][k] - n[i][k] * proj) * rstd;
        if (ds != nullptr) o[k] = o[k] + r[i][k];
      }
      store8f(dx + base + c * 8, o);
      if (ddelta != nullptr) store8h(ddelta + base + c * 8, o);
    }
  }
}

// Element-granular variants for hidden sizes that are not a multiple of 8 or unaligned buffers.
__global__ void rmsnorm_fwd_any(const float *x, const uint16_t *delta, const float *w,
                                float *s_out, uint16_t *y, float *ypad, const int64_t *pad_idx,
                                float *rstd_out, int64_t hidden, float eps) {
  pdl_wait();
  pdl_release();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t base = row * hidden;
  float ss = 0.f;
  for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
    float v = x[base + c];
    if (delta != nullptr) {
      v = v + __half2float(__ushort_as_half(delta[base + c]));
      s_out[base + c] = v;
    }
    ss += v * v;
  }
  const float total = block_sum(ss, red);
  const float rstd = 1.0f / sqrtf(total / (float)hidden + eps);
  const int64_t dest = ypad != nullptr ? pad_idx[row] * hidden : 0;
  for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
    const float v = delta != nullptr ? s_out[base + c] : x[base + c];
    const float o = __fmul_rn(__fmul_rn(v, rstd), w[c]);
    y[base + c] = __half_as_ushort(__float2half_rn(o));
    if (ypad != nullptr) ypad[dest + c] = o;
  }
  if (threadIdx.x == 0) rstd_out[row] = rstd;
}

__global__ void rmsnorm_bwd_any(const float *s, const float *rstd_in, const float *w,
                                const uint16_t *dy, const float *dypad, const int64_t *pad_idx,
                                const float *ds, float *dx, uint16_t *ddelta, int64_t hidden) {
  pdl_wait();
  pdl_release();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t base = row * hidden;
  const int64_t src = dypad != nullptr ? pad_idx[row] * hidden : 0;
  const float rstd = rstd_in[row];
  auto grad = [&](int64_t c) {
    float g = dy != nullptr ? __half2float(__ushort_as_half(dy[base + c])) : 0.f;
    if (dypad != nullptr) g = g + dypad[src + c];
    return g * w[c];
  };
  float dot = 0.f;
  for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) dot += grad(c) * (s[base + c] * rstd);
  const float proj = block_sum(dot, red) / (float)hidden;
  for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
    const float n = s[base + c] * rstd;
    float o = (grad(c) - n * proj) * rstd;
    if (ds != nullptr) o = o + ds[base + c];
    dx[base + c] = o;
    if (ddelta != nullptr) ddelta[base + c] = __half_as_ushort(__float2half_rn(o));
  }
}

// Threads per row and chunks per thread for the vector kernels; NCH 0 = use the scalar kernel.
// Rows get more chunks per thread while the grid would not fit in one wave of resident
// threads (a second, partial wave costs a whole row-latency of its own).
void plan_rows(int64_t hidden, int64_t rows, bool vec_ok, int &threads, int &nch) {
  if (!vec_ok || hidden % 8 != 0 || hidden > 8 * 8 * 1024) {
    threads = 256;
    nch = 0;
    return;
  }
  const int64_t chunks = hidden / 8;
  int64_t t = ((chunks + 31) / 32) * 32;
  nch = 1;
  while (t > 256 && nch < 8) {
    nch *= 2;
    t = (((chunks + nch - 1) / nch + 31) / 32) * 32;
  }
  if (t > 1024) {
    threads = 256;
    nch = 0;
    return;
  }
  const int64_t resident = (int64_t)sm_count() * 2048 * 7 / 8;
  while (nch < 8 && rows * t > resident && (chunks + 2 * nch - 1) / (2 * nch) >= 32) {
    nch *= 2;
    t = (((chunks + nch - 1) / nch + 31) / 32) * 32;
  }
  threads = (int)t;
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" int tb_add_rmsnorm_fwd(const float *x, const uint16_t *delta, const float *weight,
                                  float *s_out, uint16_t *y, float *ypad, const int64_t *pad_idx,
                                  float *rstd_out, int64_t rows, int64_t hidden, float eps,
                                  void *stream) {
  if (rows < 0 || hidden <= 0) return set_error(TB_EINVAL, "add_rmsnorm_fwd: rows %lld hidden %lld",
                                                (long long)rows, (long long)hidden);
  if (!x || !weight || !y || !rstd_out)
    return set_error(TB_EINVAL, "add_rmsnorm_fwd: x, weight, y and rstd are required");
  if (delta && !s_out) return set_error(TB_EINVAL, "add_rmsnorm_fwd: delta given without s_out");
  if (ypad && !pad_idx) return set_error(TB_EINVAL, "add_rmsnorm_fwd: ypad given without pad_idx");
  if (rows == 0) return TB_OK;
  if (rows > 0x7fffffffLL) return set_error(TB_EINVAL, "add_rmsnorm_fwd: too many rows");
  const bool vec_ok = aligned(x, 16) && aligned(weight, 16) && aligned(y, 16) &&
                      (!delta || (aligned(delta, 16) && aligned(s_out, 16))) &&
                      (!ypad || aligned(ypad, 16));
  int threads, nch;
  plan_rows(hidden, rows, vec_ok, threads, nch);
  cudaStream_t st = as_stream(stream);
  const dim3 grid((unsigned)rows);
  int rc;
  switch (nch) {
    case 1: rc = launch("add_rmsnorm_fwd", rmsnorm_fwd_vec<1>, grid, threads, 0, st, x, delta, weight, s_out, y, ypad, pad_idx, rstd_out, hidden, eps); break;
    case 2: rc = launch("add_rmsnorm_fwd", rmsnorm_fwd_vec<2>, grid, threads, 0, st, x, delta, weight, s_out, y, ypad, pad_idx, rstd_out, hidden, eps); break;
    case 4: rc = launch("add_rmsnorm_fwd", rmsnorm_fwd_vec<4>, grid, threads, 0, st, x, delta, weight, s_out, y, ypad, pad_idx, rstd_out, hidden, eps); break;
    case 8: rc = launch("add_rmsnorm_fwd", rmsnorm_fwd_vec<8>, grid, threads, 0, st, x, delta, weight, s_out, y, ypad, pad_idx, rstd_out, hidden, eps); break;
    default: rc = launch("add_rmsnorm_fwd", rmsnorm_fwd_any, grid, threads, 0, st, x, delta, weight, s_out, y, ypad, pad_idx, rstd_out, hidden, eps); break;
  }
  return rc;
}

extern "C" int tb_add_rmsnorm_bwd(const float *s, const float *rstd, const float *weight,
                                  const uint16_t *dy, const float *dypad, const int64_t *pad_idx,
                                  const float *ds, float *dx, uint16_t *ddelta, int64_t rows,
                                  int64_t hidden, void *stream) {
  if (rows < 0 || hidden <= 0) return set_error(TB_EINVAL, "add_rmsnorm_bwd: rows %lld hidden %lld",
                                                (long long)rows, (long long)hidden);
  if (!s || !rstd || !weight || !dx)
    return set_error(TB_EINVAL, "add_rmsnorm_bwd: s, rstd, weight and dx are required");
  if (dypad && !pad_idx) return set_error(TB_EINVAL, "add_rmsnorm_bwd: dypad given without pad_idx");
  if (rows == 0) return TB_OK;
  if (rows > 0x7fffffffLL) return set_error(TB_EINVAL, "add_rmsnorm_bwd: too many rows");
  const bool vec_ok = aligned(s, 16) && aligned(weight, 16) && aligned(dx, 16) &&
                      (!dy || aligned(dy, 16)) && (!dypad || aligned(dypad, 16)) &&
                      (!ds || aligned(ds, 16)) && (!ddelta || aligned(ddelta, 16));
  int threads, nch;
  plan_rows(hidden, rows, vec_ok, threads, nch);
  cudaStream_t st = as_stream(stream);
  const dim3 grid((unsigned)rows);
  int rc;
  switch (nch) {
    case 1: rc = launch("add_rmsnorm_bwd", rmsnorm_bwd_vec<1>, grid, threads, 0, st, s, rstd, weight, dy, dypad, pad_idx, ds, dx, ddelta, hidden); break;
    case 2: rc = launch("add_rmsnorm_bwd", rmsnorm_bwd_vec<2>, grid, threads, 0, st, s, rstd, weight, dy, dypad, pad_idx, ds, dx, ddelta, hidden); break;
    case 4: rc = launch("add_rmsnorm_bwd", rmsnorm_bwd_vec<4>, grid, threads, 0, st, s, rstd, weight, dy, dypad, pad_idx, ds, dx, ddelta, hidden); break;
    case 8: rc = launch("add_rmsnorm_bwd", rmsnorm_bwd_vec<8>, grid, threads, 0, st, s, rstd, weight, dy, dypad, pad_idx, ds, dx, ddelta, hidden); break;
    default: rc = launch("add_rmsnorm_bwd", rmsnorm_bwd_any, grid, threads, 0, st, s, rstd, weight, dy, dypad, pad_idx, ds, dx, ddelta, hidden); break;
  }
  return rc;
}
