// The head's row bookkeeping around its GEMMs, for sm_100a: the labelled-first order of the rows
// and the return to row order of the gradient and the per-row statistics.
//
// Reference: solution/head.py:87-156 (FusedHeadLoss) gathers the labelled rows, runs the chunked
// sweeps over them and scatters the gradient back. This library's head does the same with the
// rows sorted labelled-first (a stable partition), so the dh GEMM covers a prefix of the sorted
// rows. With PyTorch ops that bookkeeping took 16 small launches per head call (flags, argsort,
// gathers, a zero fill, index_copy, the inverse permutation, three gathers and a cast); here it
// is two kernels:
//   head_order_kernel   one CTA: per-thread counts of labelled rows over contiguous row ranges,
//                       a block scan, then each row's place in the stable partition; writes
//                       order[place] = row and the sorted targets;
//   head_unsort_kernel  grad[order[i]] = dh[i] for the first `keep` sorted rows and 0 for the
//                       rest (16-byte vectors), and each row's entropy, loss and hit moved back
//                       to its own row.
#include "common.cuh"

namespace tb {
namespace {

constexpr int kOrderThreads = 1024;

__global__ void __launch_bounds__(kOrderThreads)
    head_order_kernel(const int64_t *__restrict__ targets, int64_t rows, int64_t ignore,
                      int64_t *__restrict__ order, int64_t *__restrict__ tgt_sorted) {
  pdl_wait();
  pdl_release();
  __shared__ int64_t warp_tot[kOrderThreads / 32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int64_t per = (rows + kOrderThreads - 1) / kOrderThreads;
  const int64_t r0 = min(rows, (int64_t)t * per), r1 = min(rows, r0 + per);
  int64_t mine = 0;
  for (int64_t r = r0; r < r1; ++r) mine += __ldg(targets + r) != ignore;
  // block-wide exclusive scan of the per-thread counts, in row order
  int64_t incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  int64_t before_warp = 0, total = 0;
  for (int w = 0; w < kOrderThreads / 32; ++w) {
    const int64_t v = warp_tot[w];
    if (w < warp) before_warp += v;
    total += v;
  }
  int64_t lab = before_warp + incl - mine;  // labelled rows before r0
  int64_t unl = total + (r0 - lab);         // places of the unlabelled rows before r0 come after
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t tg = __ldg(targets + r);
    const int64_t place = tg != ignore ? lab++ : unl++;
    order[place] = r;
    tgt_sorted[place] = tg;
  }
}

__global__ void __launch_bounds__(256)
    head_unsort_kernel(const int64_t *__restrict__ order, int64_t rows, int64_t keep,
                       const uint16_t *__restrict__ dh, int64_t width, uint16_t *__restrict__ grad,
                       const float *__restrict__ ent_s, const float *__restrict__ loss_s,
                       const int32_t *__restrict__ cor_s, float *__restrict__ ent,
                       float *__restrict__ loss, uint8_t *__restrict__ cor) {
  pdl_wait();
  pdl_release();
  const int64_t nvec = grad != nullptr ? width / 8 : 1;  // 16-byte vectors of a gradient row
  const int64_t n = rows * nvec;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = i / nvec, v = i - s * nvec;
    const int64_t row = __ldg(order + s);
    if (grad != nullptr) {
      uint4 val = make_uint4(0u, 0u, 0u, 0u);
      if (s < keep) val = __ldg(reinterpret_cast<const uint4 *>(dh + s * width) + v);
      reinterpret_cast<uint4 *>(grad + row * width)[v] = val;
    }
    if (v == 0) {
      ent[row] = __ldg(ent_s + s);
      loss[row] = __ldg(loss_s + s);
      cor[row] = __ldg(cor_s + s) != 0;
    }
  }
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" int tb_head_order(const int64_t *targets, int64_t rows, int64_t ignore_index,
                             int64_t *order, int64_t *targets_sorted, void *stream) {
  if (rows < 0) return set_error(TB_EINVAL, "head_order: rows %lld", (long long)rows);
  if (rows == 0) return TB_OK;
  if (!targets || !order || !targets_sorted)
    return set_error(TB_EINVAL, "head_order: targets, order and targets_sorted are required");
  return launch("head_order", head_order_kernel, dim3(1), kOrderThreads, 0, as_stream(stream),
                targets, rows, ignore_index, order, targets_sorted);
}

extern "C" int tb_head_unsort(const int64_t *order, int64_t rows, int64_t keep,
                              const uint16_t *dh_sorted, int64_t width, uint16_t *grad,
                              const float *entropy_sorted, const float *loss_sorted,
                              const int32_t *correct_sorted, float *entropy, float *loss,
                              uint8_t *correct, void *stream) {
  if (rows < 0 || keep < 0 || keep > rows || width < 0)
    return set_error(TB_EINVAL, "head_unsort: rows %lld keep %lld width %lld", (long long)rows,
                     (long long)keep, (long long)width);
  if (rows == 0) return TB_OK;
  if (!order || !entropy_sorted || !loss_sorted || !correct_sorted || !entropy || !loss ||
      !correct)
    return set_error(TB_EINVAL, "head_unsort: order and the statistics are required");
  if (grad != nullptr) {
    if (width == 0 || width % 8 || (keep > 0 && !dh_sorted))
      return set_error(TB_EINVAL, "head_unsort: width %lld (a multiple of 8) and dh for the kept rows",
                       (long long)width);
    if (!aligned(grad, 16) || (dh_sorted && !aligned(dh_sorted, 16)))
      return set_error(TB_EALIGN, "head_unsort: grad and dh must be 16-byte aligned");
  }
  const int64_t n = rows * (grad != nullptr ? width / 8 : 1);
  int64_t blocks = (n + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  return launch("head_unsort", head_unsort_kernel, dim3((unsigned)blocks), 256, 0,
                as_stream(stream), order, rows, keep, dh_sorted, width, grad, entropy_sorted,
                loss_sorted, correct_sorted, entropy, loss, correct);
}
