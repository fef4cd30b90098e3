// The glue of the LoRA branches on q_proj / v_proj around PyTorch's dropout, for sm_100a.
//
// Reference: solution/model.py:195-206 (_lora_branch): per adapter, peft's
// lora_B(lora_A(dropout(x))) * scaling on x = the padded fp32 norm output (the unpatched model's
// input, so dropout draws the same mask), then index_select of the real tokens; under fp16
// autocast lora_A's input is cast to fp16. The dropout itself stays PyTorch's (its random
// stream is what makes the fused step match the unpatched one); these two kernels replace the
// operations around it:
//   forward   tb_lora_gather:       x16[r] = fp16(dropped[pos_idx[r]])   for q and v at once
//             (index_select + the autocast cast, two launches per adapter);
//   backward  tb_lora_dropout_grad: g[p] = fp32(dxq[t]) * sq * mq[p] + fp32(dxv[t]) * sv * mv[p]
//             for t = slot_tok[p] (0 at padding), the padded gradient of the shared dropout
//             input (per adapter: zero-fill + index_add + dropout backward, then the sum of the
//             two, five launches and ~100 MB of traffic per layer at 2048 x 1536).
// Each product and the sum are rounded on their own (no contraction), as the separate PyTorch
// operations round them.
#include "common.cuh"

namespace tb {
namespace {

constexpr int kThreads = 256;

// One thread per 8 columns of one real row, grid-stride.
__global__ void __launch_bounds__(kThreads)
    lora_gather_vec(const float *__restrict__ dq, const float *__restrict__ dv,
                    const int64_t *__restrict__ pos_idx, uint16_t *__restrict__ xq,
                    uint16_t *__restrict__ xv, int64_t rows, int64_t vec_per_row) {
  const int64_t n = rows * vec_per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vec_per_row, c = (i - r * vec_per_row) * 8;
    const int64_t hidden = vec_per_row * 8;
    const int64_t src = __ldg(pos_idx + r) * hidden + c;
    float f[8];
    if (dq != nullptr) {
      load8f(dq + src, f);
      store8h(xq + r * hidden + c, f);
    }
    if (dv != nullptr) {
      load8f(dv + src, f);
      store8h(xv + r * hidden + c, f);
    }
  }
}

__global__ void lora_gather_any(const float *dq, const float *dv, const int64_t *pos_idx,
                                uint16_t *xq, uint16_t *xv, int64_t rows, int64_t hidden) {
  const int64_t n = rows * hidden;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / hidden, c = i - r * hidden;
    const int64_t src = pos_idx[r] * hidden + c;
    if (dq != nullptr) xq[i] = __half_as_ushort(__float2half_rn(dq[src]));
    if (dv != nullptr) xv[i] = __half_as_ushort(__float2half_rn(dv[src]));
  }
}

__device__ __forceinline__ float branch_grad(const uint16_t *dx, const uint8_t *mask, int64_t tok,
                                             int64_t p, int64_t c, int64_t hidden, float scale) {
  if (dx == nullptr) return 0.f;
  const float g = __half2float(__ushort_as_half(dx[tok * hidden + c]));
  if (mask == nullptr) return g;  // no dropout on this adapter
  return mask[p * hidden + c] ? __fmul_rn(g, scale) : 0.f;
}

// One thread per 8 columns of one padded slot, grid-stride; rows of padding are written zero.
__global__ void __launch_bounds__(kThreads)
    lora_dropout_grad_vec(const uint16_t *__restrict__ dxq, const uint16_t *__restrict__ dxv,
                          const uint8_t *__restrict__ mq, const uint8_t *__restrict__ mv,
                          const int32_t *__restrict__ slot_tok, float *__restrict__ g,
                          int64_t slots, int64_t vec_per_row, float sq, float sv) {
  const int64_t n = slots * vec_per_row;
  const int64_t hidden = vec_per_row * 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i / vec_per_row, c = (i - p * vec_per_row) * 8;
    const int64_t tok = __ldg(slot_tok + p);
    float out[8];
    if (tok < 0) {
#pragma unroll
      for (int k = 0; k < 8; ++k) out[k] = 0.f;
    } else {
      float a[8], b[8];
      uint2 ma = make_uint2(0x01010101u, 0x01010101u), mb = ma;
      if (dxq != nullptr) {
        load8h(dxq + tok * hidden + c, a);
        if (mq != nullptr) ma = __ldg(reinterpret_cast<const uint2 *>(mq + p * hidden + c));
      }
      if (dxv != nullptr) {
        load8h(dxv + tok * hidden + c, b);
        if (mv != nullptr) mb = __ldg(reinterpret_cast<const uint2 *>(mv + p * hidden + c));
      }
      const uint8_t *bytes_a = reinterpret_cast<const uint8_t *>(&ma);
      const uint8_t *bytes_b = reinterpret_cast<const uint8_t *>(&mb);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float ga = dxq == nullptr ? 0.f
                         : mq == nullptr ? a[k]
                                         : (bytes_a[k] ? __fmul_rn(a[k], sq) : 0.f);
        const float gb = dxv == nullptr ? 0.f
                         : mv == nullptr ? b[k]
                                         : (bytes_b[k] ? __fmul_rn(b[k], sv) : 0.f);
        out[k] = __fadd_rn(ga, gb);
      }
    }
    store8f(g + p * hidden + c, out);
  }
}

__global__ void lora_dropout_grad_any(const uint16_t *dxq, const uint16_t *dxv, const uint8_t *mq,
                                      const uint8_t *mv, const int32_t *slot_tok, float *g,
                                      int64_t slots, int64_t hidden, float sq, float sv) {
  const int64_t n = slots * hidden;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i / hidden, c = i - p * hidden;
    const int64_t tok = slot_tok[p];
    if (tok < 0) {
      g[i] = 0.f;
      continue;
    }
    g[i] = __fadd_rn(branch_grad(dxq, mq, tok, p, c, hidden, sq),
                     branch_grad(dxv, mv, tok, p, c, hidden, sv));
  }
}

unsigned grid_for(int64_t n) {
  int64_t blocks = (n + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  return (unsigned)(blocks > 0 ? blocks : 1);
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" int tb_lora_gather(const float *dropped_q, const float *dropped_v,
                              const int64_t *pos_idx, uint16_t *xq, uint16_t *xv, int64_t rows,
                              int64_t hidden, void *stream) {
  if (rows < 0 || hidden <= 0)
    return set_error(TB_EINVAL, "lora_gather: rows %lld hidden %lld", (long long)rows,
                     (long long)hidden);
  if (rows == 0) return TB_OK;
  if (!pos_idx || (!dropped_q && !dropped_v) || (dropped_q && !xq) || (dropped_v && !xv))
    return set_error(TB_EINVAL, "lora_gather: pos_idx and a (dropped, x16) pair are required");
  cudaStream_t st = as_stream(stream);
  const bool vec = hidden % 8 == 0 && (!dropped_q || (aligned(dropped_q, 16) && aligned(xq, 16))) &&
                   (!dropped_v || (aligned(dropped_v, 16) && aligned(xv, 16)));
  if (vec) {
    lora_gather_vec<<<grid_for(rows * hidden / 8), kThreads, 0, st>>>(dropped_q, dropped_v,
                                                                       pos_idx, xq, xv, rows,
                                                                       hidden / 8);
  } else {
    lora_gather_any<<<grid_for(rows * hidden), kThreads, 0, st>>>(dropped_q, dropped_v, pos_idx,
                                                                  xq, xv, rows, hidden);
  }
  return check_launch("lora_gather");
}

extern "C" int tb_lora_dropout_grad(const uint16_t *dxq, const uint16_t *dxv,
                                    const uint8_t *mask_q, const uint8_t *mask_v,
                                    const int32_t *slot_tok, float *grad, int64_t slots,
                                    int64_t hidden, float scale_q, float scale_v, void *stream) {
  if (slots < 0 || hidden <= 0)
    return set_error(TB_EINVAL, "lora_dropout_grad: slots %lld hidden %lld", (long long)slots,
                     (long long)hidden);
  if (slots == 0) return TB_OK;
  if (!slot_tok || !grad)
    return set_error(TB_EINVAL, "lora_dropout_grad: slot_tok and grad are required");
  cudaStream_t st = as_stream(stream);
  const bool vec = hidden % 8 == 0 && aligned(grad, 16) && (!dxq || aligned(dxq, 16)) &&
                   (!dxv || aligned(dxv, 16)) && (!mask_q || aligned(mask_q, 8)) &&
                   (!mask_v || aligned(mask_v, 8));
  if (vec) {
    lora_dropout_grad_vec<<<grid_for(slots * hidden / 8), kThreads, 0, st>>>(
        dxq, dxv, mask_q, mask_v, slot_tok, grad, slots, hidden / 8, scale_q, scale_v);
  } else {
    lora_dropout_grad_any<<<grid_for(slots * hidden), kThreads, 0, st>>>(
        dxq, dxv, mask_q, mask_v, slot_tok, grad, slots, hidden, scale_q, scale_v);
  }
  return check_launch("lora_dropout_grad");
}
