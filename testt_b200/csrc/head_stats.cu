// Vocabulary head statistics and in-place dlogits over a chunk of fp16 logits, for sm_100a.
//
// Reference: solution/head.py:34-76 (head_stats_grad_kernel) and its launch :108-110. One CTA of
// 512 threads per row, as many rows resident per SM as fit. Sweep 1 is an online softmax per
// thread (running max, sum of e^(z-m), sum of e^(z-m) z and the first argmax) over 16-byte
// vectors of 8 logits, four vectors in flight per thread, followed by a shuffle + shared-memory
// merge of the per-thread states. Sweep 2 (labelled rows only) rewrites the row in place with
// fp16((exp(z - lse) - [c == target]) * grad_scale). Rounding: z are the fp16 logits widened to
// fp32, exactly as the reference reads them; exponentials use the fast __expf that the
// reference's tl.exp lowers to.
#include <math_constants.h>

#include "common.cuh"

namespace tb {
namespace {

constexpr int kThreads = 512;
constexpr int kUnroll = 4;

struct Online {
  float m, s, dz, best;
  int64_t idx;
};

__device__ __forceinline__ void online_add(Online &o, float z, int64_t c) {
  if (z > o.best) {
    o.best = z;
    o.idx = c;
  }
  if (z > o.m) {
    const float r = __expf(o.m - z);  // 0 when o.m is -inf
    o.s *= r;
    o.dz *= r;
    o.m = z;
  }
  const float e = __expf(z - o.m);
  o.s += e;
  o.dz += e * z;
}

__device__ __forceinline__ Online online_merge(const Online &a, const Online &b) {
  Online o;
  o.m = fmaxf(a.m, b.m);
  const float ra = a.m == -CUDART_INF_F ? 0.f : __expf(a.m - o.m);
  const float rb = b.m == -CUDART_INF_F ? 0.f : __expf(b.m - o.m);
  o.s = a.s * ra + b.s * rb;
  o.dz = a.dz * ra + b.dz * rb;
  const bool take_b = b.best > a.best || (b.best == a.best && b.idx < a.idx);
  o.best = take_b ? b.best : a.best;
  o.idx = take_b ? b.idx : a.idx;
  return o;
}

__device__ __forceinline__ Online shfl_online(const Online &a, int off) {
  Online b;
  b.m = __shfl_xor_sync(0xffffffffu, a.m, off);
  b.s = __shfl_xor_sync(0xffffffffu, a.s, off);
  b.dz = __shfl_xor_sync(0xffffffffu, a.dz, off);
  b.best = __shfl_xor_sync(0xffffffffu, a.best, off);
  b.idx = __shfl_xor_sync(0xffffffffu, a.idx, off);
  return b;
}

__global__ void __launch_bounds__(kThreads)
    head_stats_grad_rows(uint16_t *__restrict__ logits, const int64_t *__restrict__ targets,
                         float *__restrict__ entropy, float *__restrict__ loss,
                         int32_t *__restrict__ correct, int64_t vocab, int64_t ld,
                         float grad_scale, bool vec) {
  __shared__ Online part[kThreads / 32];
  __shared__ float lse_sh;
  const int64_t row = blockIdx.x;
  uint16_t *base = logits + row * ld;
  const int64_t target = __ldg(targets + row);
  const bool labelled = target != -100 && target >= 0 && target < vocab;

  Online o{-CUDART_INF_F, 0.f, 0.f, -CUDART_INF_F, 0x7fffffffffffffffLL};
  const int64_t nvec = vec ? vocab / 8 : 0;
  for (int64_t v0 = threadIdx.x; v0 < nvec; v0 += (int64_t)kThreads * kUnroll) {
    float z[kUnroll][8];
#pragma unroll
    for (int r = 0; r < kUnroll; ++r) {
      const int64_t v = v0 + (int64_t)r * kThreads;
      if (v < nvec) load8h_rw(base + v * 8, z[r]);
    }
#pragma unroll
    for (int r = 0; r < kUnroll; ++r) {
      const int64_t v = v0 + (int64_t)r * kThreads;
      if (v < nvec) {
        float lm = z[r][0];
#pragma unroll
        for (int k = 1; k < 8; ++k) lm = fmaxf(lm, z[r][k]);
        if (lm > o.m) {
          const float sc = __expf(o.m - lm);
          o.s *= sc;
          o.dz *= sc;
          o.m = lm;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float e = __expf(z[r][k] - o.m);
          o.s += e;
          o.dz += e * z[r][k];
          if (z[r][k] > o.best) {
            o.best = z[r][k];
            o.idx = v * 8 + k;
          }
        }
      }
    }
  }
  for (int64_t c = nvec * 8 + threadIdx.x; c < vocab; c += kThreads)
    online_add(o, __half2float(__ushort_as_half(base[c])), c);

#pragma unroll
  for (int off = 16; off > 0; off >>= 1) o = online_merge(o, shfl_online(o, off));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) part[warp] = o;
  __syncthreads();
  if (warp == 0) {
    o = lane < kThreads / 32 ? part[lane]
                             : Online{-CUDART_INF_F, 0.f, 0.f, -CUDART_INF_F, 0x7fffffffffffffffLL};
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) o = online_merge(o, shfl_online(o, off));
    if (lane == 0) {
      const float lse = o.m + logf(o.s);
      entropy[row] = lse - o.dz / o.s;
      const float zt = labelled ? __half2float(__ushort_as_half(base[target])) : 0.f;
      loss[row] = labelled ? lse - zt : 0.f;
      correct[row] = (labelled && o.idx == target) ? 1 : 0;
      lse_sh = lse;
    }
  }
  __syncthreads();
  if (!labelled) return;
  const float lse = lse_sh;
  for (int64_t v0 = threadIdx.x; v0 < nvec; v0 += (int64_t)kThreads * kUnroll) {
    float z[kUnroll][8];
#pragma unroll
    for (int r = 0; r < kUnroll; ++r) {
      const int64_t v = v0 + (int64_t)r * kThreads;
      if (v < nvec) load8h_rw(base + v * 8, z[r]);
    }
#pragma unroll
    for (int r = 0; r < kUnroll; ++r) {
      const int64_t v = v0 + (int64_t)r * kThreads;
      if (v < nvec) {
        float g[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float hot = (v * 8 + k == target) ? 1.f : 0.f;
          g[k] = (__expf(z[r][k] - lse) - hot) * grad_scale;
        }
        store8h(base + v * 8, g);
      }
    }
  }
  for (int64_t c = nvec * 8 + threadIdx.x; c < vocab; c += kThreads) {
    const float z = __half2float(__ushort_as_half(base[c]));
    const float g = (__expf(z - lse) - (c == target ? 1.f : 0.f)) * grad_scale;
    base[c] = __half_as_ushort(__float2half_rn(g));
  }
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" int tb_head_stats_grad(uint16_t *logits, const int64_t *targets, float *entropy,
                                  float *loss, int32_t *correct, int64_t rows, int64_t vocab,
                                  int64_t ld, float grad_scale, void *stream) {
  if (rows < 0 || vocab <= 0 || ld < vocab)
    return set_error(TB_EINVAL, "head_stats_grad: rows %lld vocab %lld ld %lld", (long long)rows,
                     (long long)vocab, (long long)ld);
  if (rows == 0) return TB_OK;
  if (!logits || !targets || !entropy || !loss || !correct)
    return set_error(TB_EINVAL, "head_stats_grad: all pointers are required");
  if (rows > 0x7fffffffLL) return set_error(TB_EINVAL, "head_stats_grad: too many rows");
  const bool vec = aligned(logits, 16) && ld % 8 == 0;
  head_stats_grad_rows<<<(unsigned)rows, kThreads, 0, as_stream(stream)>>>(
      logits, targets, entropy, loss, correct, vocab, ld, grad_scale, vec);
  return check_launch("head_stats_grad");
}
