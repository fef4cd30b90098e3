// The token embedding of the real tokens, for sm_100a: out[r] = fp32(table[ids[pos_idx[r]]]).
//
// Reference: solution/model.py:220-225 runs the model's embedding on the padded ids; the fused
// path embeds only the real tokens. With PyTorch ops that is three launches (index_select of
// the ids, the embedding gather, the cast to the fp32 residual stream); here it is one. A thread
// takes 8 consecutive values of a row: one 16-byte load of fp16, two 16-byte stores of fp32.
// A token id outside [0, vocab) is not read: its row is written as zeros and counted in
// tb_embed_invalid_ids (PyTorch's embedding stops the device instead).
#include "common.cuh"

namespace tb {
namespace {

__device__ unsigned int g_embed_invalid = 0;

__global__ void __launch_bounds__(256)
    embed_rows_kernel(const int64_t *__restrict__ ids, const int64_t *__restrict__ pos_idx,
                      const uint16_t *__restrict__ table, float *__restrict__ out, int64_t rows,
                      int64_t hidden, int64_t vocab) {
  pdl_wait();
  pdl_release();
  const int64_t nvec = hidden / 8;
  const int64_t n = rows * nvec;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nvec, v = i - r * nvec;
    const int64_t id = __ldg(ids + __ldg(pos_idx + r));
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (id >= 0 && id < vocab) {
      load8h(table + id * hidden + v * 8, f);
    } else if (v == 0) {
      atomicAdd(&g_embed_invalid, 1u);
    }
    store8f(out + r * hidden + v * 8, f);
  }
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" int tb_embed_rows(const int64_t *ids, const int64_t *pos_idx, const uint16_t *table,
                             float *out, int64_t rows, int64_t hidden, int64_t vocab,
                             void *stream) {
  if (rows < 0 || hidden <= 0 || vocab <= 0)
    return set_error(TB_EINVAL, "embed_rows: rows %lld hidden %lld vocab %lld", (long long)rows,
                     (long long)hidden, (long long)vocab);
  if (rows == 0) return TB_OK;
  if (!ids || !pos_idx || !table || !out)
    return set_error(TB_EINVAL, "embed_rows: ids, pos_idx, table and out are required");
  if (hidden % 8)
    return set_error(TB_EINVAL, "embed_rows: hidden %lld (a multiple of 8)", (long long)hidden);
  if (!aligned(table, 16) || !aligned(out, 16))
    return set_error(TB_EALIGN, "embed_rows: table and out must be 16-byte aligned");
  const int64_t n = rows * (hidden / 8);
  int64_t blocks = (n + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  return launch("embed_rows", embed_rows_kernel, dim3((unsigned)blocks), 256, 0,
                as_stream(stream), ids, pos_idx, table, out, rows, hidden, vocab);
}

extern "C" int64_t tb_embed_invalid_ids(void) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_embed_invalid, sizeof(v)) != cudaSuccess) {
    (void)cudaGetLastError();
    return -1;
  }
  return (int64_t)v;
}
