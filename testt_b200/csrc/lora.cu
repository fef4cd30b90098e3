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

// ---- the adapters' forward in one kernel (rank 16) -------------------------------------------
// Per real row m and adapter (blockIdx.y: 0 = q, 1 = v), one warp:
//   x16 = fp16(dropped[pos_idx[m]])                         (index_select + the autocast cast)
//   h16 = fp16(x16 . fp16(A)^T)                               (lora_A, fp16 GEMM output)
//   out = fp16(fp32(fp16(h16 . fp16(B)^T)) * scaling)          (lora_B, then * scaling)
// with fp32 accumulation, the fp16 weights (the autocast casts, made by the caller) staged in
// shared memory (B transposed), the 16 sums of h reduced across the warp by a butterfly (every
// lane ends with all of them). x16 and h16 are written for the backward GEMMs.
constexpr int kRank = 16;

struct LoraFwdAdapter {
  const float *dropped;  // fp32 [slots, hidden]
  const uint16_t *a;     // fp16(lora_A weight) [16, hidden]
  const uint16_t *b;     // fp16(lora_B weight) [hout, 16]
  uint16_t *x16;         // fp16 [rows, hidden]
  uint16_t *h16;         // fp16 [rows, 16]
  uint16_t *out;         // fp16 [rows, hout]
  int hout;
  float scale;
};

struct LoraFwdArgs {
  LoraFwdAdapter ad[2];
  const int64_t *pos_idx;
  int64_t rows, rows_per_cta;
  int hidden;
};

__device__ __forceinline__ void unpack8(const uint4 v, float (&f)[8]) {
  const float2 a = unpack_half2(v.x), b = unpack_half2(v.y), c = unpack_half2(v.z),
               d = unpack_half2(v.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

__global__ void __launch_bounds__(kThreads) lora_fwd_kernel(const __grid_constant__ LoraFwdArgs a) {
  extern __shared__ __align__(16) uint8_t lora_smem[];
  const LoraFwdAdapter &p = a.ad[blockIdx.y];
  if (p.a == nullptr) return;
  const int H = a.hidden, HO = p.hout;
  uint16_t *a16 = reinterpret_cast<uint16_t *>(lora_smem);  // [16][H]
  uint16_t *bt16 = a16 + kRank * H;                          // [16][HO]: B transposed
  {
    const uint4 *src = reinterpret_cast<const uint4 *>(p.a);
    uint4 *dst = reinterpret_cast<uint4 *>(a16);
#pragma unroll 4
    for (int i = threadIdx.x; i < kRank * H / 8; i += blockDim.x) dst[i] = __ldg(src + i);
  }
#pragma unroll 2
  for (int n = threadIdx.x; n < HO; n += blockDim.x) {  // row n of B: 16 halves, 2 loads
    const uint4 lo = __ldg(reinterpret_cast<const uint4 *>(p.b + (int64_t)n * kRank));
    const uint4 hi = __ldg(reinterpret_cast<const uint4 *>(p.b + (int64_t)n * kRank + 8));
    const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
    for (int j = 0; j < kRank; ++j)
      bt16[j * HO + n] = (uint16_t)(w[j / 2] >> (16 * (j & 1)));
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int64_t m0 = (int64_t)blockIdx.x * a.rows_per_cta;
  const int64_t m1 = m0 + a.rows_per_cta < a.rows ? m0 + a.rows_per_cta : a.rows;
  for (int64_t m = m0 + warp; m < m1; m += nwarps) {
    const float *xrow = p.dropped + __ldg(a.pos_idx + m) * H;
    float acc[kRank];
#pragma unroll
    for (int j = 0; j < kRank; ++j) acc[j] = 0.f;
    for (int v = lane; v < H / 8; v += 32) {
      float x[8];
      load8f(xrow + v * 8, x);
      uint4 xv;
      xv.x = pack_half2(x[0], x[1]);
      xv.y = pack_half2(x[2], x[3]);
      xv.z = pack_half2(x[4], x[5]);
      xv.w = pack_half2(x[6], x[7]);
      *reinterpret_cast<uint4 *>(p.x16 + m * H + v * 8) = xv;
      unpack8(xv, x);
#pragma unroll
      for (int j = 0; j < kRank; ++j) {
        float w[8];
        unpack8(*reinterpret_cast<const uint4 *>(a16 + j * H + v * 8), w);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[j] = fmaf(x[e], w[e], acc[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < kRank; ++j) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], off);
    }
    float h[kRank];
    uint32_t hp[kRank / 2];
#pragma unroll
    for (int j = 0; j < kRank; j += 2) {
      hp[j / 2] = pack_half2(acc[j], acc[j + 1]);
      const float2 r = unpack_half2(hp[j / 2]);
      h[j] = r.x;
      h[j + 1] = r.y;
    }
    if (lane < 2) {
      const uint4 hv = lane == 0 ? make_uint4(hp[0], hp[1], hp[2], hp[3])
                                 : make_uint4(hp[4], hp[5], hp[6], hp[7]);
      *reinterpret_cast<uint4 *>(p.h16 + m * kRank + lane * 8) = hv;
    }
    for (int v = lane; v < HO / 8; v += 32) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = 0.f;
#pragma unroll
      for (int j = 0; j < kRank; ++j) {
        float w[8];
        unpack8(*reinterpret_cast<const uint4 *>(bt16 + j * HO + v * 8), w);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = fmaf(h[j], w[e], o[e]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e)  // the GEMM's fp16 output, then * scaling (rounded on store)
        o[e] = __half2float(__float2half_rn(o[e])) * p.scale;
      store8h(p.out + m * HO + v * 8, o);
    }
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

extern "C" int tb_lora_forward(const float *dropped_q, const uint16_t *a_q, const uint16_t *b_q,
                               uint16_t *x16_q, uint16_t *h16_q, uint16_t *out_q, int64_t hout_q,
                               float scale_q, const float *dropped_v, const uint16_t *a_v,
                               const uint16_t *b_v, uint16_t *x16_v, uint16_t *h16_v,
                               uint16_t *out_v, int64_t hout_v, float scale_v,
                               const int64_t *pos_idx, int64_t rows, int64_t hidden, int32_t rank,
                               void *stream) {
  if (rank != kRank)
    return set_error(TB_EINVAL, "lora_forward: rank %d (the fused kernel takes rank %d)", rank,
                     kRank);
  if (rows < 0 || hidden <= 0 || hidden % 8 || hout_q % 8 || hout_v % 8 || hout_q < 0 ||
      hout_v < 0 || hidden > 8192 || hout_q > 8192 || hout_v > 8192)
    return set_error(TB_EINVAL, "lora_forward: rows %lld hidden %lld hout %lld/%lld",
                     (long long)rows, (long long)hidden, (long long)hout_q, (long long)hout_v);
  if (rows == 0 || (!a_q && !a_v)) return TB_OK;
  if (!pos_idx) return set_error(TB_EINVAL, "lora_forward: pos_idx is required");
  LoraFwdArgs args{};
  const float *dr[2] = {dropped_q, dropped_v};
  const uint16_t *aa[2] = {a_q, a_v}, *bb[2] = {b_q, b_v};
  uint16_t *xx[2] = {x16_q, x16_v}, *hh[2] = {h16_q, h16_v}, *oo[2] = {out_q, out_v};
  const int64_t ho[2] = {hout_q, hout_v};
  const float sc[2] = {scale_q, scale_v};
  int64_t max_hout = 0;
  for (int i = 0; i < 2; ++i) {
    if (aa[i] == nullptr) continue;
    if (!dr[i] || !bb[i] || !xx[i] || !hh[i] || !oo[i])
      return set_error(TB_EINVAL, "lora_forward: adapter %d needs dropped, a, b, x16, h16, out", i);
    if (!aligned(dr[i], 16) || !aligned(xx[i], 16) || !aligned(hh[i], 16) || !aligned(oo[i], 16) ||
        !aligned(aa[i], 16) || !aligned(bb[i], 16))
      return set_error(TB_EALIGN, "lora_forward: 16-byte aligned buffers are required");
    args.ad[i] = LoraFwdAdapter{dr[i], aa[i], bb[i], xx[i], hh[i], oo[i], (int)ho[i], sc[i]};
    if (ho[i] > max_hout) max_hout = ho[i];
  }
  args.pos_idx = pos_idx;
  args.rows = rows;
  args.hidden = (int)hidden;
  // about one CTA per SM over both adapters, 8 warps each
  int64_t ctas = sm_count() / 2;
  if (ctas * (kThreads / 32) > rows) ctas = (rows + kThreads / 32 - 1) / (kThreads / 32);
  if (ctas < 1) ctas = 1;
  args.rows_per_cta = (rows + ctas - 1) / ctas;
  ctas = (rows + args.rows_per_cta - 1) / args.rows_per_cta;
  const size_t smem = (size_t)kRank * (hidden + max_hout) * 2;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(lora_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return check_launch("lora_forward attribute");
  lora_fwd_kernel<<<dim3((unsigned)ctas, 2), kThreads, smem, as_stream(stream)>>>(args);
  return check_launch("lora_forward");
}
