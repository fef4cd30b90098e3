// Vocabulary head statistics and in-place dlogits over a chunk of fp16 logits, for sm_100a.
//
// Reference: solution/head.py:34-76 (head_stats_grad_kernel) and its launch :108-110. One CTA of
// 512 threads per row, as many rows resident per SM as fit. Sweep 1 is an online softmax per
// thread (running max, sum of e^(z-m), sum of e^(z-m) z and the first argmax) over 16-byte
// vectors of 8 logits, four vectors in flight per thread, followed by a shuffle + shared-memory
// merge of the per-thread states. Sweep 2 (labelled rows only) rewrites the row in place with
// fp16((exp(z - lse) - [c == target]) * grad_scale). Rounding: z are the fp16 logits widened to
// fp32, exactly as the reference reads them; exponentials are the MUFU 2^x that the fast exp of
// the reference's tl.exp lowers to, with the max (or lse) shift folded into the FFMA forming its
// argument. Per logit: one max, one FFMA + ex2, one add, one FFMA in sweep 1 (the first argmax
// is searched only in a vector that raises the running max), one FFMA + ex2 + multiply in sweep
// 2 (the one-hot term only in the vector holding the target).
#include <math_constants.h>

#include <mutex>

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

constexpr float kLog2e = 1.4426950408889634f;

// 2^x on the MUFU (PTX ex2.approx); e^x is taken as 2^(x log2 e), with the shift by the
// running max folded into one FFMA: e^(z - m) = 2^(z log2e - m log2e)
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Folds 8 consecutive logits (columns c0 .. c0 + 7) into the state. The running max is also the
// best value; the first index of a new maximum is searched only when the max grows (a tie with
// an earlier maximum keeps the earlier index: the first argmax).
__device__ __forceinline__ void online_add8(Online &o, const float (&z)[8], int64_t c0) {
  float lm = z[0];
#pragma unroll
  for (int k = 1; k < 8; ++k) lm = fmaxf(lm, z[k]);
  if (lm > o.m) {
    const float sc = ex2f((o.m - lm) * kLog2e);  // 0 while m is -inf
    o.s *= sc;
    o.dz *= sc;
    o.m = lm;
    o.best = lm;
    int first = 7;
#pragma unroll
    for (int k = 6; k >= 0; --k)
      if (z[k] == lm) first = k;
    o.idx = c0 + first;
  }
  const float ml = o.m * kLog2e;
  float s0 = 0.f, s1 = 0.f, d0 = 0.f, d1 = 0.f;
#pragma unroll
  for (int k = 0; k < 8; k += 2) {
    const float e0 = ex2f(fmaf(z[k], kLog2e, -ml));
    const float e1 = ex2f(fmaf(z[k + 1], kLog2e, -ml));
    s0 += e0;
    s1 += e1;
    d0 = fmaf(e0, z[k], d0);
    d1 = fmaf(e1, z[k + 1], d1);
  }
  o.s += s0 + s1;
  o.dz += d0 + d1;
}

// fp16((e^(z - lse) - [column == target]) * scale) of 8 consecutive logits (columns c0 ..),
// in place; nl = -lse log2 e. The target test runs only in the one vector that holds it.
__device__ __forceinline__ void dlogits8(uint16_t *p, const float (&z)[8], float nl,
                                         int64_t c0, int64_t target, float scale) {
  float g[8];
  if ((uint64_t)(target - c0) < 8u) {
#pragma unroll
    for (int k = 0; k < 8; ++k)
      g[k] = (ex2f(fmaf(z[k], kLog2e, nl)) - (c0 + k == target ? 1.f : 0.f)) * scale;
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) g[k] = ex2f(fmaf(z[k], kLog2e, nl)) * scale;
  }
  store8h(p, g);
}

__global__ void __launch_bounds__(kThreads)
    head_stats_grad_rows(uint16_t *__restrict__ logits, const int64_t *__restrict__ targets,
                         float *__restrict__ entropy, float *__restrict__ loss,
                         int32_t *__restrict__ correct, int64_t vocab, int64_t ld,
                         float grad_scale, bool vec) {
  pdl_wait();
  pdl_release();
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
      if (v < nvec) online_add8(o, z[r], v * 8);
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
  const float nl = -lse * kLog2e;
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
      if (v < nvec) dlogits8(base + v * 8, z[r], nl, v * 8, target, grad_scale);
    }
  }
  for (int64_t c = nvec * 8 + threadIdx.x; c < vocab; c += kThreads) {
    const float z = __half2float(__ushort_as_half(base[c]));
    const float g = (__expf(z - lse) - (c == target ? 1.f : 0.f)) * grad_scale;
    base[c] = __half_as_ushort(__float2half_rn(g));
  }
}


// ---- split form: partials over column ranges, a merge, and the dlogits sweep ----------------
// The same two sweeps as head_stats_grad_rows, split so that one row can be spread over several
// CTAs (more parallelism for short chunks) and over several GPUs (a vocabulary-sharded head):
// each (row, column range) yields a partial online-softmax state, states of one row are merged
// in any grouping (max, rescaled sums, first argmax on ties), and the dlogits sweep then needs
// only the merged lse.

constexpr int kPartThreads = 256;
constexpr int kPartFields = 6;  // max, sum e, sum e z, best value, z[target], target found

__device__ __forceinline__ void block_merge(Online &o, Online *sh) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) o = online_merge(o, shfl_online(o, off));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sh[warp] = o;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    o = lane < nw ? sh[lane] : Online{-CUDART_INF_F, 0.f, 0.f, -CUDART_INF_F, 0x7fffffffffffffffLL};
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) o = online_merge(o, shfl_online(o, off));
  }
}

__global__ void __launch_bounds__(kPartThreads)
    head_partials_kernel(const uint16_t *__restrict__ logits, const int64_t *__restrict__ targets,
                         float *__restrict__ part, int64_t *__restrict__ part_idx, int64_t cols,
                         int64_t ld, int64_t col_offset, int64_t chunk, bool vec) {
  pdl_wait();
  pdl_release();
  __shared__ Online sh[kPartThreads / 32];
  const int64_t row = blockIdx.y;
  const int split = blockIdx.x, splits = gridDim.x;
  const int64_t lo = (int64_t)split * chunk;
  const int64_t hi = lo + chunk < cols ? lo + chunk : cols;
  const uint16_t *base = logits + row * ld;
  const int64_t target = __ldg(targets + row);
  Online o{-CUDART_INF_F, 0.f, 0.f, -CUDART_INF_F, 0x7fffffffffffffffLL};
  int64_t vlo = lo, vend = lo;
  if (vec && lo < hi) {
    vend = lo + ((hi - lo) / 8) * 8;
    for (int64_t c0 = lo + threadIdx.x * 8; c0 < vend; c0 += (int64_t)kPartThreads * 8 * kUnroll) {
      float z[kUnroll][8];
#pragma unroll
      for (int r = 0; r < kUnroll; ++r) {
        const int64_t c = c0 + (int64_t)r * kPartThreads * 8;
        if (c < vend) load8h(base + c, z[r]);
      }
#pragma unroll
      for (int r = 0; r < kUnroll; ++r) {
        const int64_t c = c0 + (int64_t)r * kPartThreads * 8;
        if (c < vend) online_add8(o, z[r], col_offset + c);
      }
    }
    vlo = vend;
  }
  for (int64_t c = vlo + threadIdx.x; c < hi; c += kPartThreads)
    online_add(o, __half2float(__ushort_as_half(base[c])), col_offset + c);
  block_merge(o, sh);
  if (threadIdx.x == 0) {
    float *out = part + (row * splits + split) * kPartFields;
    out[0] = o.m;
    out[1] = o.s;
    out[2] = o.dz;
    out[3] = o.best;
    const bool found = target >= col_offset + lo && target < col_offset + hi;
    out[4] = found ? __half2float(__ushort_as_half(base[target - col_offset])) : 0.f;
    out[5] = found ? 1.f : 0.f;
    part_idx[row * splits + split] = o.idx;
  }
}

// One warp per row over n_groups x splits partial states laid out [group][row][split].
__global__ void head_merge_kernel(const float *__restrict__ part,
                                  const int64_t *__restrict__ part_idx,
                                  const int64_t *__restrict__ targets, int64_t rows, int n_groups,
                                  int splits, float *__restrict__ lse_out,
                                  float *__restrict__ entropy, float *__restrict__ loss,
                                  int32_t *__restrict__ correct) {
  pdl_wait();
  pdl_release();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  Online o{-CUDART_INF_F, 0.f, 0.f, -CUDART_INF_F, 0x7fffffffffffffffLL};
  float zt = 0.f, found = 0.f;
  const int n = n_groups * splits;
  // a lane merges states lane, lane + 32, ... in that order; four states' loads are issued
  // before they are merged (a row has hundreds of states: one load round trip per state made
  // this a chain of latencies)
  constexpr int kAhead = 4;
  int p = lane;
  for (; p + 32 * (kAhead - 1) < n; p += 32 * kAhead) {
    Online b[kAhead];
    float zq[kAhead], fq[kAhead];
#pragma unroll
    for (int k = 0; k < kAhead; ++k) {
      const int pk = p + 32 * k;
      const int g = pk / splits, sp = pk - g * splits;
      const int64_t at = ((int64_t)g * rows + row) * splits + sp;
      const float *q = part + at * kPartFields;
      b[k] = Online{__ldg(q), __ldg(q + 1), __ldg(q + 2), __ldg(q + 3), __ldg(part_idx + at)};
      zq[k] = __ldg(q + 4);
      fq[k] = __ldg(q + 5);
    }
#pragma unroll
    for (int k = 0; k < kAhead; ++k) {
      o = online_merge(o, b[k]);
      if (fq[k] != 0.f && found == 0.f) {
        zt = zq[k];
        found = 1.f;
      }
    }
  }
  for (; p < n; p += 32) {
    const int g = p / splits, sp = p - g * splits;
    const int64_t at = ((int64_t)g * rows + row) * splits + sp;
    const float *q = part + at * kPartFields;
    Online b{q[0], q[1], q[2], q[3], part_idx[at]};
    o = online_merge(o, b);
    if (q[5] != 0.f && found == 0.f) {
      zt = q[4];
      found = 1.f;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    o = online_merge(o, shfl_online(o, off));
    const float zo = __shfl_xor_sync(0xffffffffu, zt, off);
    const float fo = __shfl_xor_sync(0xffffffffu, found, off);
    if (found == 0.f && fo != 0.f) {
      zt = zo;
      found = fo;
    }
  }
  if (lane == 0) {
    const int64_t target = targets[row];
    const bool labelled = target != -100 && found != 0.f;
    const float lse = o.m + logf(o.s);
    lse_out[row] = lse;
    entropy[row] = lse - o.dz / o.s;
    loss[row] = labelled ? lse - zt : 0.f;
    correct[row] = (labelled && o.idx == target) ? 1 : 0;
  }
}

// One warp per (row, output split): the row's input partial states [lo, hi) of its splits_in
// states (contiguous per row) merged into one, every argmax index shifted by col_offset (a
// vocabulary shard's first column); the target field is taken from the state that holds it.
__global__ void head_fold_kernel(const float *__restrict__ part,
                                 const int64_t *__restrict__ part_idx, int64_t rows,
                                 int splits_in, int splits_out, int64_t col_offset,
                                 float *__restrict__ out, int64_t *__restrict__ out_idx) {
  pdl_wait();
  pdl_release();
  const int lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= rows * splits_out) return;
  const int64_t row = w / splits_out;
  const int o = (int)(w - row * splits_out);
  const int per = (splits_in + splits_out - 1) / splits_out;
  const int lo = o * per, hi = min(splits_in, lo + per);
  constexpr int64_t kNone = 0x7fffffffffffffffLL;
  Online acc{-CUDART_INF_F, 0.f, 0.f, -CUDART_INF_F, kNone};
  float zt = 0.f, found = 0.f;
  for (int p = lo + lane; p < hi; p += 32) {
    const int64_t at = row * splits_in + p;
    const float *q = part + at * kPartFields;
    const int64_t ix = part_idx[at];
    const Online b{q[0], q[1], q[2], q[3], ix == kNone ? kNone : ix + col_offset};
    acc = online_merge(acc, b);
    if (q[5] != 0.f && found == 0.f) {
      zt = q[4];
      found = 1.f;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    acc = online_merge(acc, shfl_online(acc, off));
    const float zo = __shfl_xor_sync(0xffffffffu, zt, off);
    const float fo = __shfl_xor_sync(0xffffffffu, found, off);
    if (found == 0.f && fo != 0.f) {
      zt = zo;
      found = fo;
    }
  }
  if (lane == 0) {
    float *q = out + w * kPartFields;
    q[0] = acc.m;
    q[1] = acc.s;
    q[2] = acc.dz;
    q[3] = acc.best;
    q[4] = found != 0.f ? zt : 0.f;
    q[5] = found;
    out_idx[w] = acc.idx;
  }
}

// dlogits over labelled rows, in place: flat over 8-value vectors (n < 2^32 vectors).
__global__ void __launch_bounds__(256)
    head_dlogits_kernel(uint16_t *__restrict__ logits, const int64_t *__restrict__ targets,
                        const float *__restrict__ lse, uint32_t n, FastDiv vpr, int64_t ld,
                        int64_t col_offset, float grad_scale) {
  pdl_wait();
  pdl_release();
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    uint32_t row, v;
    vpr.divmod(i, row, v);
    const int64_t target = __ldg(targets + row);
    if (target == -100) continue;
    const float nl = -__ldg(lse + row) * kLog2e;
    uint16_t *p = logits + (int64_t)row * ld + (int64_t)v * 8;
    float z[8];
    load8h_rw(p, z);
    dlogits8(p, z, nl, col_offset + (int64_t)v * 8, target, grad_scale);
  }
}

__global__ void head_dlogits_any(uint16_t *logits, const int64_t *targets, const float *lse,
                                 int64_t rows, int64_t cols, int64_t ld, int64_t col_offset,
                                 float grad_scale) {
  pdl_wait();
  pdl_release();
  const int64_t n = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / cols, c = i - row * cols;
    const int64_t target = targets[row];
    if (target == -100) continue;
    uint16_t *p = logits + row * ld + c;
    const float z = __half2float(__ushort_as_half(*p));
    const float g = (__expf(z - lse[row]) - (col_offset + c == target ? 1.f : 0.f)) * grad_scale;
    *p = __half_as_ushort(__float2half_rn(g));
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
  return launch("head_stats_grad", head_stats_grad_rows, (unsigned)rows, kThreads, 0,
                as_stream(stream), logits, targets, entropy, loss, correct, vocab, ld, grad_scale,
                vec);
}

extern "C" int tb_head_partials(const uint16_t *logits, const int64_t *targets, float *part,
                                int64_t *part_idx, int64_t rows, int64_t cols, int64_t ld,
                                int64_t col_offset, int32_t splits, void *stream) {
  if (rows < 0 || cols <= 0 || ld < cols || splits < 1 || col_offset < 0)
    return set_error(TB_EINVAL, "head_partials: rows %lld cols %lld ld %lld splits %d",
                     (long long)rows, (long long)cols, (long long)ld, splits);
  if (rows == 0) return TB_OK;
  if (!logits || !targets || !part || !part_idx)
    return set_error(TB_EINVAL, "head_partials: all pointers are required");
  if (rows > 65535) return set_error(TB_EINVAL, "head_partials: at most 65535 rows per call");
  const bool vec = aligned(logits, 16) && ld % 8 == 0;
  int64_t chunk = (cols + splits - 1) / splits;
  chunk = ((chunk + 7) / 8) * 8;
  const dim3 grid((unsigned)splits, (unsigned)rows);
  return launch("head_partials", head_partials_kernel, grid, kPartThreads, 0, as_stream(stream),
                logits, targets, part, part_idx, cols, ld, col_offset, chunk, vec);
}

extern "C" int tb_head_merge(const float *part, const int64_t *part_idx, const int64_t *targets,
                             int64_t rows, int32_t n_groups, int32_t splits, float *lse,
                             float *entropy, float *loss, int32_t *correct, void *stream) {
  if (rows < 0 || n_groups < 1 || splits < 1)
    return set_error(TB_EINVAL, "head_merge: rows %lld groups %d splits %d", (long long)rows,
                     n_groups, splits);
  if (rows == 0) return TB_OK;
  if (!part || !part_idx || !targets || !lse || !entropy || !loss || !correct)
    return set_error(TB_EINVAL, "head_merge: all pointers are required");
  const int warps = 8;
  const unsigned blocks = (unsigned)((rows + warps - 1) / warps);
  return launch("head_merge", head_merge_kernel, blocks, warps * 32, 0, as_stream(stream), part,
                part_idx, targets, rows, n_groups, splits, lse, entropy, loss, correct);
}

extern "C" int tb_head_fold(const float *part, const int64_t *part_idx, int64_t rows,
                            int32_t splits_in, int64_t col_offset, int32_t splits_out,
                            float *part_out, int64_t *idx_out, void *stream) {
  if (rows < 0 || splits_in < 1 || splits_out < 1 || splits_out > splits_in || col_offset < 0)
    return set_error(TB_EINVAL, "head_fold: rows %lld splits %d -> %d offset %lld",
                     (long long)rows, splits_in, splits_out, (long long)col_offset);
  if (rows == 0) return TB_OK;
  if (!part || !part_idx || !part_out || !idx_out)
    return set_error(TB_EINVAL, "head_fold: all pointers are required");
  const int64_t warps = rows * splits_out;
  const int per_block = 8;
  if ((warps + per_block - 1) / per_block > 0x7fffffffLL)
    return set_error(TB_EINVAL, "head_fold: too many rows");
  return launch("head_fold", head_fold_kernel, (unsigned)((warps + per_block - 1) / per_block),
                per_block * 32, 0, as_stream(stream), part, part_idx, rows, (int)splits_in,
                (int)splits_out, col_offset, part_out, idx_out);
}

extern "C" int tb_head_dlogits(uint16_t *logits, const int64_t *targets, const float *lse,
                               int64_t rows, int64_t cols, int64_t ld, int64_t col_offset,
                               float grad_scale, void *stream) {
  if (rows < 0 || cols <= 0 || ld < cols || col_offset < 0)
    return set_error(TB_EINVAL, "head_dlogits: rows %lld cols %lld ld %lld", (long long)rows,
                     (long long)cols, (long long)ld);
  if (rows == 0) return TB_OK;
  if (!logits || !targets || !lse) return set_error(TB_EINVAL, "head_dlogits: all pointers are required");
  cudaStream_t st = as_stream(stream);
  const int64_t nvec = rows * (cols / 8);
  const int64_t cap = (int64_t)sm_count() * 8;
  if (cols % 8 == 0 && ld % 8 == 0 && aligned(logits, 16) && nvec < (1LL << 31)) {
    int64_t blocks = (nvec + 255) / 256;
    if (blocks > cap) blocks = cap;
    return launch("head_dlogits", head_dlogits_kernel, (unsigned)blocks, 256, 0, st, logits,
                  targets, lse, (uint32_t)nvec, FastDiv((uint32_t)(cols / 8)), ld, col_offset,
                  grad_scale);
  }
  int64_t blocks = (rows * cols + 255) / 256;
  if (blocks > cap) blocks = cap;
  return launch("head_dlogits", head_dlogits_any, (unsigned)blocks, 256, 0, st, logits, targets,
                lse, rows, cols, ld, col_offset, grad_scale);
}

// ---- the same statistics with no allocation anywhere (tb_head_stats_grad_noalloc) -----------
// Scratch of the split form (partial states, their argmax indices, the merged lse) lives in one
// file-scope device array instead of caller-provided buffers. Each GPU that loads the library
// holds it (1,179,648 bytes) until the process exits. Every call shares it and leaves the last
// call's contents behind; nothing in it needs to start at zero (the partials kernel writes every
// (row, split) state before the merge reads it, the merge writes every lse before the dlogits
// sweep reads it). Calls whose kernels overlap on the GPU (on different streams) race on it.
namespace tb {
namespace {

constexpr int64_t kNoAllocMaxRows = 32768;   // rows per call
constexpr int64_t kNoAllocMaxParts = 32768;  // rows x splits per call
constexpr size_t kNoAllocPartBytes = (size_t)kNoAllocMaxParts * kPartFields * sizeof(float);
constexpr size_t kNoAllocIdxBytes = (size_t)kNoAllocMaxParts * sizeof(int64_t);
constexpr size_t kNoAllocLseBytes = (size_t)kNoAllocMaxRows * sizeof(float);
constexpr size_t kNoAllocBytes = kNoAllocPartBytes + kNoAllocIdxBytes + kNoAllocLseBytes;

static __device__ __align__(256) unsigned char g_head_scratch[kNoAllocBytes];

// Device address of g_head_scratch on the current device (the host-side name of the array is
// not a device address). Outside stream capture it is looked up on every call (cheap), so a
// device reset between calls, which reloads the library's module, never leaves a stale
// address behind; during capture, where the lookup could load the module, the address taken by
// an earlier call on the device is used (hence: a first call before any capture).
int head_scratch(cudaStream_t stream, unsigned char **out) {
  static std::mutex lock;
  static unsigned char *cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return set_error(TB_EDEVICE, "head_stats_grad_noalloc: no usable current device");
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &capture) != cudaSuccess) {
    (void)cudaGetLastError();
    capture = cudaStreamCaptureStatusActive;  // unknown: do not risk a lookup
  }
  std::lock_guard<std::mutex> guard(lock);
  if (capture == cudaStreamCaptureStatusNone || cached[dev] == nullptr) {
    if (capture != cudaStreamCaptureStatusNone)
      return set_error(TB_EINVAL, "head_stats_grad_noalloc: the first call on a device must "
                       "come before any stream capture");
    void *ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_head_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return set_error(TB_ELAUNCH, "head_stats_grad_noalloc: scratch address: %s",
                       cudaGetErrorString(e));
    cached[dev] = static_cast<unsigned char *>(ptr);
  }
  *out = cached[dev];
  return TB_OK;
}

}  // namespace
}  // namespace tb

extern "C" int tb_head_stats_grad_noalloc(uint16_t *logits, const int64_t *targets,
                                          float *entropy, float *loss, int32_t *correct,
                                          int64_t rows, int64_t vocab, int64_t ld,
                                          float grad_scale, void *stream) {
  if (rows < 0 || vocab <= 0 || ld < vocab)
    return set_error(TB_EINVAL, "head_stats_grad_noalloc: rows %lld vocab %lld ld %lld",
                     (long long)rows, (long long)vocab, (long long)ld);
  if (rows > kNoAllocMaxRows)
    return set_error(TB_EINVAL,
                     "head_stats_grad_noalloc: %lld rows exceed the fixed scratch (at most %lld "
                     "rows per call; split the call or use tb_head_stats_grad)",
                     (long long)rows, (long long)kNoAllocMaxRows);
  if (rows == 0) return TB_OK;
  if (!logits || !targets || !entropy || !loss || !correct)
    return set_error(TB_EINVAL, "head_stats_grad_noalloc: all pointers are required");
  unsigned char *scratch = nullptr;
  int rc = head_scratch(as_stream(stream), &scratch);
  if (rc != TB_OK) return rc;
  float *part = reinterpret_cast<float *>(scratch);
  int64_t *part_idx = reinterpret_cast<int64_t *>(scratch + kNoAllocPartBytes);
  float *lse = reinterpret_cast<float *>(scratch + kNoAllocPartBytes + kNoAllocIdxBytes);
  // enough (row, split) CTAs to fill the GPU, within the scratch
  int64_t splits = (4LL * sm_count() + rows - 1) / rows;
  if (splits > 16) splits = 16;
  if (splits > kNoAllocMaxParts / rows) splits = kNoAllocMaxParts / rows;
  if (splits < 1) splits = 1;
  rc = tb_head_partials(logits, targets, part, part_idx, rows, vocab, ld, 0, (int32_t)splits,
                        stream);
  if (rc != TB_OK) return rc;
  rc = tb_head_merge(part, part_idx, targets, rows, 1, (int32_t)splits, lse, entropy, loss,
                     correct, stream);
  if (rc != TB_OK) return rc;
  return tb_head_dlogits(logits, targets, lse, rows, vocab, ld, 0, grad_scale, stream);
}
