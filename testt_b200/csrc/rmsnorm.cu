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
#include <algorithm>

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

// dy is fp16 [rows, hidden], or (dyp non-NULL) the fp32 K-split partial products of the GEMM
// that produces it, nparts of them pstride elements apart: summed in part order and rounded to
// fp16 once, the GEMM's fp16 output (the split-K reduction folded into this kernel).
template <int NCH>
__global__ void rmsnorm_bwd_vec(const float *__restrict__ s, const float *__restrict__ rstd_in,
                                const float *__restrict__ w, const uint16_t *__restrict__ dy,
                                const float *__restrict__ dyp, int nparts, int64_t pstride,
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
      if (dyp != nullptr) {
        load8f(dyp + base + c * 8, g[i]);
        for (int p = 1; p < nparts; ++p) {
          float q[8];
          load8f(dyp + p * pstride + base + c * 8, q);
#pragma unroll
          for (int k = 0; k < 8; ++k) g[i][k] = g[i][k] + q[k];
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) g[i][k] = __half2float(__float2half_rn(g[i][k]));
      } else if (dy != nullptr) {
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

// ---- backward with the LoRA branch's input gradient formed in place ---------------------------
// The padded-layout gradient dypad that rmsnorm_bwd_vec reads is, on the fused path, the dropout
// backward of the two rank-16 adapters (q and v) fed by this norm's padded output:
//   dypad[slot(row), c] = drop_q'(fp16(dh_q[row] . a16_q[:, c])) + drop_v'(fp16(dh_v[row] . a16_v[:, c]))
// with drop'(x) = mask ? x * scale : 0 (x when the adapter has no mask). This kernel computes that
// sum per element in registers, with the operations and roundings of lora_dropout_grad_expand
// (sixteen fmaf in rank order from 0, the fp16 rounding of the GEMM output, the masked scale, the
// q + v sum), instead of reading it from an fp32 [slots, hidden] tensor another launch wrote.
// The rest is rmsnorm_bwd_vec's arithmetic with its thread -> chunk mapping and reduction order
// (as long as plan_rows gives it one or two chunks per thread, which covers the step's row
// counts), so the outputs are the two-launch path's, bit for bit. A CTA takes R rows: every
// thread reads its columns of both fp16(A) (16 ranks x 8 columns each, L2-resident) once for
// all R rows.
struct RmsLoraBranch {
  const uint16_t *dh;    // fp16 [rows, 16], the adapter's h gradient (NULL: adapter absent)
  const uint16_t *a16;   // fp16 [16, hidden], the adapter's lora_A weight as autocast cast it
  const uint8_t *mask;   // bool [slots, hidden] dropout keep-mask (NULL: no dropout)
  float scale;           // 1 / (1 - p)
};

struct RmsLoraArgs {
  const float *s, *rstd, *w;
  const uint16_t *dy;      // fp16 [rows, hidden] gradient of y (NULL: none)
  const int64_t *pad_idx;  // slot of each row
  const float *ds;         // fp32 [rows, hidden] residual gradient (NULL: none)
  float *dx;
  uint16_t *ddelta;        // NULL: not wanted
  RmsLoraBranch br[2];
  int64_t rows, hidden;
};

// registers per thread for NCH chunks and R rows (the launcher uses two chunks of one row, for
// 2056-4096 columns): 112, three CTAs of up to 192 threads per SM
template <int NCH, int R>
constexpr int rms_lora_regs() {
  return NCH * R == 1 ? 64 : NCH * R == 2 ? 112 : 128;
}

template <int NCH, int R>
__global__ void __maxnreg__((rms_lora_regs<NCH, R>()))
    rmsnorm_bwd_lora_vec(const __grid_constant__ RmsLoraArgs a) {
  pdl_wait();
  pdl_release();
  __shared__ float red[R][32];
  __shared__ float dh_sh[R][2][16];  // the rows' dh of both adapters (the same for every thread)
  const int nch = (int)(a.hidden / 8);
  const int64_t row0 = (int64_t)blockIdx.x * R;
  float g[R][NCH][8], n[R][NCH][8], r[R][NCH][8], wv[NCH][8];
  uint2 mk[R][2][NCH];
  float rstd[R];
  bool rv[R];
  if (threadIdx.x < R * 2 * 2) {  // one 8-value half of one row's dh each
    const int i = threadIdx.x >> 2, ad = (threadIdx.x >> 1) & 1, half = threadIdx.x & 1;
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (row0 + i < a.rows && a.br[ad].dh != nullptr)
      load8h(a.br[ad].dh + (row0 + i) * 16 + half * 8, f);
#pragma unroll
    for (int k = 0; k < 8; ++k) dh_sh[i][ad][half * 8 + k] = f[k];
  }
  // every load of the R rows is issued before the expansion and the reductions
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int64_t row = row0 + i;
    rv[i] = row < a.rows;
    const int64_t base = row * a.hidden;
    const int64_t slot = rv[i] ? __ldg(a.pad_idx + row) : 0;
    rstd[i] = rv[i] ? __ldg(a.rstd + row) : 0.f;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int c = threadIdx.x + j * blockDim.x;
#pragma unroll
      for (int k = 0; k < 8; ++k) g[i][j][k] = n[i][j][k] = r[i][j][k] = 0.f;
#pragma unroll
      for (int ad = 0; ad < 2; ++ad) mk[i][ad][j] = make_uint2(0x01010101u, 0x01010101u);
      if (!rv[i] || c >= nch) continue;
      if (a.dy != nullptr) load8h(a.dy + base + c * 8, g[i][j]);
      if (a.ds != nullptr) load8f(a.ds + base + c * 8, r[i][j]);
      load8f(a.s + base + c * 8, n[i][j]);
#pragma unroll
      for (int ad = 0; ad < 2; ++ad)
        if (a.br[ad].dh != nullptr && a.br[ad].mask != nullptr)
          mk[i][ad][j] = __ldg(reinterpret_cast<const uint2 *>(a.br[ad].mask + slot * a.hidden + c * 8));
    }
  }
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int c = threadIdx.x + j * blockDim.x;
    if (c < nch) load8f(a.w + c * 8, wv[j]);
  }
  __syncthreads();  // dh_sh written
  // the LoRA input gradient of each row's 8 columns, added to dy's
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int c = threadIdx.x + j * blockDim.x;
    if (c >= nch) continue;
    float p[R][8];
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
      for (int k = 0; k < 8; ++k) p[i][k] = 0.f;
#pragma unroll
    for (int ad = 0; ad < 2; ++ad) {
      const RmsLoraBranch &b = a.br[ad];
      if (b.dh == nullptr) continue;
      float acc[R][8];
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[i][k] = 0.f;
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const uint4 av4 = __ldg(reinterpret_cast<const uint4 *>(b.a16 + (int64_t)q * a.hidden + c * 8));
        const uint32_t aw[4] = {av4.x, av4.y, av4.z, av4.w};
#pragma unroll
        for (int i = 0; i < R; ++i) {
          const float hf = dh_sh[i][ad][q];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = unpack_half2(aw[e]);
            acc[i][2 * e] = fmaf(hf, f.x, acc[i][2 * e]);
            acc[i][2 * e + 1] = fmaf(hf, f.y, acc[i][2 * e + 1]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const uint2 m = mk[i][ad][j];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float dxk = __half2float(__float2half_rn(acc[i][k]));  // the fp16 GEMM output
          const uint32_t keep = ((k < 4 ? m.x : m.y) >> (8 * (k & 3))) & 0xffu;
          const float gk = b.mask == nullptr ? dxk : (keep ? __fmul_rn(dxk, b.scale) : 0.f);
          p[i][k] = ad == 0 ? gk : __fadd_rn(p[i][k], gk);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
      for (int k = 0; k < 8; ++k) g[i][j][k] = g[i][j][k] + p[i][k];
  }
  float dot[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    dot[i] = 0.f;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int c = threadIdx.x + j * blockDim.x;
      if (c < nch) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          g[i][j][k] = g[i][j][k] * wv[j][k];
          n[i][j][k] = n[i][j][k] * rstd[i];
          dot[i] += g[i][j][k] * n[i][j][k];
        }
      }
    }
  }
  // block_sum's order for each row: butterfly within the warp, then over the warps' sums
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const float v = warp_sum(dot[i]);
    if (lane == 0) red[i][warp] = v;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < R; ++i) {
    if (!rv[i]) continue;
    const float proj = warp_sum(lane < nwarps ? red[i][lane] : 0.f) / (float)a.hidden;
    const int64_t base = (row0 + i) * a.hidden;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int c = threadIdx.x + j * blockDim.x;
      if (c < nch) {
        float o[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          o[k] = (g[i][j][k] - n[i][j][k] * proj) * rstd[i];
          if (a.ds != nullptr) o[k] = o[k] + r[i][j][k];
        }
        store8f(a.dx + base + c * 8, o);
        if (a.ddelta != nullptr) store8h(a.ddelta + base + c * 8, o);
      }
    }
  }
}

// The same backward for up to 192 chunks of 8 columns (hidden <= 1536), reading fp16(A) once per
// launch. A thread takes half a chunk (4 columns; lanes 2i and 2i + 1 share chunk i) and keeps
// its columns of both adapters' A as fp32 (16 ranks x 4 columns x 2 adapters, 128 registers)
// for the whole launch, so the expansion is 64 packed fp32 FMAs per row and no conversion. CTAs
// loop over rows blockIdx.x, + gridDim.x, ... (about 4 rows per CTA at 621 rows, one CTA per
// SM). A row's inputs (dy, s, ds, both masks, each thread its own 4 columns; the two dh rows and
// rstd) are copied by cp.async into a ring of kRowStages shared-memory stages, kRowStages - 1
// rows ahead of the row being computed; the slots of the first kRowStages rows are loaded side
// by side, and each later row's slot one loop iteration before its copies are issued.
// Every value is rmsnorm_bwd_lora_vec's: the expansion's fmaf chains per column (fma.rn.f32x2
// rounds each lane as fmaf), and the row sum in the plain kernel's order: lane 2i + 1 continues
// lane 2i's FMA chain over the chunk's first 4 columns, the chunk sums go through shared memory,
// and the warps that hold them in the plain kernel's layout (32 chunks each) reduce them by the
// same butterfly, then across warps as block_sum does.
constexpr int kRowStages = 4;
constexpr int kRowsMaxChunks = 192;

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async8(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// bytes of one ring stage for T threads: s [T] x 16, ds [T] x 16, dy [T] x 8, masks [2][T] x 4,
// the two dh rows (64), rstd (4, padded to 16)
__host__ __device__ constexpr int row_stage_bytes(int T) { return 48 * T + 80; }

__global__ void __launch_bounds__(2 * kRowsMaxChunks, 1)
    rmsnorm_bwd_lora_rows(const __grid_constant__ RmsLoraArgs a) {
  pdl_wait();
  pdl_release();
  extern __shared__ __align__(16) uint8_t ring[];
  __shared__ float red[32];
  __shared__ float chunk_dot[kRowsMaxChunks];
  const int T = blockDim.x;
  const int stage_bytes = row_stage_bytes(T);
  const int nch = (int)(a.hidden / 8);
  const int t = threadIdx.x, chunk = t >> 1, half = t & 1;
  const int col = chunk * 8 + half * 4;  // this thread's first column
  const bool live = chunk < nch;
  const int lane = t & 31, warp = t >> 5;
  const int plain_warps = (nch + 31) >> 5;  // the plain kernel's warps (32 chunks each)
  const int64_t stride = gridDim.x;
  const int o_ds = 16 * T, o_dy = 32 * T, o_m = 40 * T, o_dh = 48 * T, o_rstd = 48 * T + 64;

  // one row's copies into a stage, committed as one group (an empty group past the last row)
  auto issue = [&](int64_t row, int64_t slot, int stage) {
    uint8_t *st = ring + (size_t)stage * stage_bytes;
    if (row < a.rows) {
      const int64_t base = row * a.hidden + col;
      if (live) {
        cp_async16(st + 16 * t, a.s + base);
        if (a.ds != nullptr) cp_async16(st + o_ds + 16 * t, a.ds + base);
        if (a.dy != nullptr) cp_async8(st + o_dy + 8 * t, a.dy + base);
#pragma unroll
        for (int ad = 0; ad < 2; ++ad)
          if (a.br[ad].dh != nullptr && a.br[ad].mask != nullptr)
            cp_async4(st + o_m + 4 * (ad * T + t), a.br[ad].mask + slot * a.hidden + col);
      }
      if (t < 4 && a.br[t >> 1].dh != nullptr)  // one 8-value half of one adapter's dh row
        cp_async16(st + o_dh + 16 * t, a.br[t >> 1].dh + row * 16 + (t & 1) * 8);
      if (t == 4) cp_async4(st + o_rstd, a.rstd + row);
    }
    cp_async_commit();
  };

  // the slots of the first kRowStages rows, loaded side by side; the first kRowStages - 1 rows'
  // copies; after that, each row's slot is loaded one loop iteration before its copies
  const int64_t r0 = blockIdx.x;
  int64_t slot_ahead;
  {
    int64_t sl[kRowStages];
#pragma unroll
    for (int k = 0; k < kRowStages; ++k)
      sl[k] = r0 + k * stride < a.rows ? __ldg(a.pad_idx + r0 + k * stride) : 0;
#pragma unroll
    for (int k = 0; k < kRowStages - 1; ++k) issue(r0 + k * stride, sl[k], k);
    slot_ahead = sl[kRowStages - 1];
  }

  // this thread's 4 columns of both fp16(A), as fp32, for every row
  float2 af[2][16][2];
#pragma unroll
  for (int ad = 0; ad < 2; ++ad)
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      uint2 v = make_uint2(0u, 0u);
      if (live && a.br[ad].dh != nullptr)
        v = __ldg(reinterpret_cast<const uint2 *>(a.br[ad].a16 + (int64_t)q * a.hidden + col));
      af[ad][q][0] = unpack_half2(v.x);
      af[ad][q][1] = unpack_half2(v.y);
    }

  int stage = 0;
  for (int64_t row = r0; row < a.rows; row += stride) {
    {
      const int64_t ahead = row + (kRowStages - 1) * stride;
      issue(ahead, slot_ahead, stage == 0 ? kRowStages - 1 : stage - 1);
      slot_ahead = ahead + stride < a.rows ? __ldg(a.pad_idx + ahead + stride) : 0;
    }
    cp_async_wait<kRowStages - 1>();  // this thread's copies of `row`
    __syncthreads();                  // and the dh rows and rstd other threads copied
    const uint8_t *st = ring + (size_t)stage * stage_bytes;
    const float rstd = *reinterpret_cast<const float *>(st + o_rstd);
    float g[4] = {0.f, 0.f, 0.f, 0.f}, n[4] = {0.f, 0.f, 0.f, 0.f};
    if (live) {
      if (a.dy != nullptr) {
        const uint2 v = *reinterpret_cast<const uint2 *>(st + o_dy + 8 * t);
        const float2 f0 = unpack_half2(v.x), f1 = unpack_half2(v.y);
        g[0] = f0.x; g[1] = f0.y; g[2] = f1.x; g[3] = f1.y;
      }
      float p[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ad = 0; ad < 2; ++ad) {
        const RmsLoraBranch &b = a.br[ad];
        if (b.dh == nullptr) continue;
        const uint4 *dh4 = reinterpret_cast<const uint4 *>(st + o_dh + 32 * ad);
        const uint4 h0 = dh4[0], h1 = dh4[1];
        const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float2 hf2 = unpack_half2(hw[q >> 1]);
          const float hf = (q & 1) ? hf2.y : hf2.x;
          acc0 = __ffma2_rn(make_float2(hf, hf), af[ad][q][0], acc0);
          acc1 = __ffma2_rn(make_float2(hf, hf), af[ad][q][1], acc1);
        }
        const float acc[4] = {acc0.x, acc0.y, acc1.x, acc1.y};
        const uint32_t m = b.mask != nullptr
                               ? *reinterpret_cast<const uint32_t *>(st + o_m + 4 * (ad * T + t))
                               : 0x01010101u;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float dxk = __half2float(__float2half_rn(acc[k]));  // the fp16 GEMM output
          const uint32_t keep = (m >> (8 * k)) & 0xffu;
          const float gk = b.mask == nullptr ? dxk : (keep ? __fmul_rn(dxk, b.scale) : 0.f);
          p[k] = ad == 0 ? gk : __fadd_rn(p[k], gk);
        }
      }
      const float4 w4 = __ldg(reinterpret_cast<const float4 *>(a.w + col));
      const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
      const float4 s4 = *reinterpret_cast<const float4 *>(st + 16 * t);
      n[0] = s4.x; n[1] = s4.y; n[2] = s4.z; n[3] = s4.w;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        g[k] = g[k] + p[k];
        g[k] = g[k] * wv[k];
        n[k] = n[k] * rstd;
      }
    }
    // the chunk's FMA chain across the pair: lane 2i runs columns 0..3 from 0, lane 2i + 1 runs
    // columns 4..7 from lane 2i's result
    float part = 0.f;
    if (live && !half) {
#pragma unroll
      for (int k = 0; k < 4; ++k) part += g[k] * n[k];
    }
    const float from_even = __shfl_up_sync(0xffffffffu, part, 1);  // every lane of the warp
    if (live && half) {
      float dot = from_even;
#pragma unroll
      for (int k = 0; k < 4; ++k) dot += g[k] * n[k];
      chunk_dot[chunk] = dot;
    }
    __syncthreads();  // every chunk's sum
    if (warp < plain_warps) {
      const int ch = warp * 32 + lane;
      const float v = warp_sum(ch < nch ? chunk_dot[ch] : 0.f);
      if (lane == 0) red[warp] = v;
    }
    __syncthreads();
    const float proj = warp_sum(lane < plain_warps ? red[lane] : 0.f) / (float)a.hidden;
    if (live) {
      const float4 s4 = *reinterpret_cast<const float4 *>(st + 16 * t);
      const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
      float r[4] = {0.f, 0.f, 0.f, 0.f};
      if (a.ds != nullptr) {
        const float4 d4 = *reinterpret_cast<const float4 *>(st + o_ds + 16 * t);
        r[0] = d4.x; r[1] = d4.y; r[2] = d4.z; r[3] = d4.w;
      }
      float o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float nk = sv[k] * rstd;
        o[k] = (g[k] - nk * proj) * rstd;
        if (a.ds != nullptr) o[k] = o[k] + r[k];
      }
      const int64_t base = row * a.hidden + col;
      *reinterpret_cast<float4 *>(a.dx + base) = make_float4(o[0], o[1], o[2], o[3]);
      if (a.ddelta != nullptr)
        *reinterpret_cast<uint2 *>(a.ddelta + base) =
            make_uint2(pack_half2(o[0], o[1]), pack_half2(o[2], o[3]));
    }
    stage = stage + 1 == kRowStages ? 0 : stage + 1;
  }
  cp_async_wait<0>();  // no copy left in flight into shared memory as the CTA ends
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

template <int NCH, int R>
int launch_rms_lora(const RmsLoraArgs &a, int threads, cudaStream_t st) {
  return launch("add_rmsnorm_bwd_lora", rmsnorm_bwd_lora_vec<NCH, R>,
                dim3((unsigned)((a.rows + R - 1) / R)), threads, 0, st, a);
}

// the row-loop kernel: its shared-memory ring (once per process: the attribute is the
// function's), and one CTA per resident slot, at most one per row
int launch_rms_lora_rows(const RmsLoraArgs &a, cudaStream_t st) {
  const int threads = (int)((2 * (a.hidden / 8) + 31) / 32 * 32);  // two threads a chunk
  const size_t smem = (size_t)kRowStages * row_stage_bytes(threads);
  // set on every call: the attribute belongs to the current device
  if (cudaFuncSetAttribute(rmsnorm_bwd_lora_rows, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)((size_t)kRowStages * row_stage_bytes(2 * kRowsMaxChunks))) !=
      cudaSuccess) {
    (void)cudaGetLastError();
    return set_error(TB_ELAUNCH, "add_rmsnorm_bwd_lora: shared memory attribute refused");
  }
  const int64_t grid = std::min<int64_t>(a.rows, resident_blocks(rmsnorm_bwd_lora_rows, threads, smem));
  return launch("add_rmsnorm_bwd_lora", rmsnorm_bwd_lora_rows, dim3((unsigned)grid), threads, smem,
                st, a);
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

namespace tb {
namespace {

// tb_add_rmsnorm_bwd with dy given either as fp16 or as nparts fp32 K-split partials
int rmsnorm_bwd_launch(const char *what, const float *s, const float *rstd, const float *weight,
                       const uint16_t *dy, const float *dyp, int nparts, int64_t pstride,
                       const float *dypad, const int64_t *pad_idx, const float *ds, float *dx,
                       uint16_t *ddelta, int64_t rows, int64_t hidden, void *stream) {
  if (rows < 0 || hidden <= 0)
    return set_error(TB_EINVAL, "%s: rows %lld hidden %lld", what, (long long)rows,
                     (long long)hidden);
  if (!s || !rstd || !weight || !dx)
    return set_error(TB_EINVAL, "%s: s, rstd, weight and dx are required", what);
  if (dypad && !pad_idx) return set_error(TB_EINVAL, "%s: dypad given without pad_idx", what);
  if (rows == 0) return TB_OK;
  if (rows > 0x7fffffffLL) return set_error(TB_EINVAL, "%s: too many rows", what);
  const bool vec_ok = aligned(s, 16) && aligned(weight, 16) && aligned(dx, 16) &&
                      (!dy || aligned(dy, 16)) && (!dyp || aligned(dyp, 16)) &&
                      (!dypad || aligned(dypad, 16)) && (!ds || aligned(ds, 16)) &&
                      (!ddelta || aligned(ddelta, 16));
  int threads, nch;
  plan_rows(hidden, rows, vec_ok, threads, nch);
  if (dyp != nullptr && nch == 0)
    return set_error(vec_ok ? TB_EINVAL : TB_EALIGN,
                     "%s: the partial-sum form needs hidden a multiple of 8 and 16-byte aligned "
                     "buffers", what);
  cudaStream_t st = as_stream(stream);
  const dim3 grid((unsigned)rows);
  switch (nch) {
    case 1: return launch(what, rmsnorm_bwd_vec<1>, grid, threads, 0, st, s, rstd, weight, dy, dyp, nparts, pstride, dypad, pad_idx, ds, dx, ddelta, hidden);
    case 2: return launch(what, rmsnorm_bwd_vec<2>, grid, threads, 0, st, s, rstd, weight, dy, dyp, nparts, pstride, dypad, pad_idx, ds, dx, ddelta, hidden);
    case 4: return launch(what, rmsnorm_bwd_vec<4>, grid, threads, 0, st, s, rstd, weight, dy, dyp, nparts, pstride, dypad, pad_idx, ds, dx, ddelta, hidden);
    case 8: return launch(what, rmsnorm_bwd_vec<8>, grid, threads, 0, st, s, rstd, weight, dy, dyp, nparts, pstride, dypad, pad_idx, ds, dx, ddelta, hidden);
    default: return launch(what, rmsnorm_bwd_any, grid, threads, 0, st, s, rstd, weight, dy, dypad, pad_idx, ds, dx, ddelta, hidden);
  }
}

}  // namespace
}  // namespace tb

extern "C" int tb_add_rmsnorm_bwd(const float *s, const float *rstd, const float *weight,
                                  const uint16_t *dy, const float *dypad, const int64_t *pad_idx,
                                  const float *ds, float *dx, uint16_t *ddelta, int64_t rows,
                                  int64_t hidden, void *stream) {
  return rmsnorm_bwd_launch("add_rmsnorm_bwd", s, rstd, weight, dy, nullptr, 0, 0, dypad, pad_idx,
                            ds, dx, ddelta, rows, hidden, stream);
}

extern "C" int tb_add_rmsnorm_bwd_parts(const float *s, const float *rstd, const float *weight,
                                        const float *dy_parts, int32_t n_parts,
                                        int64_t part_stride, const float *ds, float *dx,
                                        uint16_t *ddelta, int64_t rows, int64_t hidden,
                                        void *stream) {
  if (!dy_parts || n_parts < 1 || n_parts > 64 || part_stride < rows * hidden)
    return set_error(TB_EINVAL, "add_rmsnorm_bwd_parts: %d parts %lld elements apart", n_parts,
                     (long long)part_stride);
  if (part_stride % 4)
    return set_error(TB_EALIGN, "add_rmsnorm_bwd_parts: part stride %lld not a multiple of 4",
                     (long long)part_stride);
  return rmsnorm_bwd_launch("add_rmsnorm_bwd_parts", s, rstd, weight, nullptr, dy_parts, n_parts,
                            part_stride, nullptr, nullptr, ds, dx, ddelta, rows, hidden, stream);
}

extern "C" int tb_add_rmsnorm_bwd_lora(const float *s, const float *rstd, const float *weight,
                                       const uint16_t *dy, const int64_t *pad_idx,
                                       const float *ds, const uint16_t *dh_q,
                                       const uint16_t *a16_q, const uint8_t *mask_q,
                                       float scale_q, const uint16_t *dh_v,
                                       const uint16_t *a16_v, const uint8_t *mask_v,
                                       float scale_v, float *dx, uint16_t *ddelta, int64_t rows,
                                       int64_t hidden, int32_t rank, void *stream) {
  if (rows < 0 || hidden <= 0)
    return set_error(TB_EINVAL, "add_rmsnorm_bwd_lora: rows %lld hidden %lld", (long long)rows,
                     (long long)hidden);
  if (rank != 16)
    return set_error(TB_EINVAL, "add_rmsnorm_bwd_lora: rank %d (the kernel takes rank 16)", rank);
  if (!s || !rstd || !weight || !dx || !pad_idx)
    return set_error(TB_EINVAL, "add_rmsnorm_bwd_lora: s, rstd, weight, dx and pad_idx are required");
  if ((dh_q && !a16_q) || (dh_v && !a16_v))
    return set_error(TB_EINVAL, "add_rmsnorm_bwd_lora: an adapter's dh needs its fp16 A");
  if (rows == 0) return TB_OK;
  if (rows > 0x7fffffffLL) return set_error(TB_EINVAL, "add_rmsnorm_bwd_lora: too many rows");
  const bool vec_ok = aligned(s, 16) && aligned(weight, 16) && aligned(dx, 16) &&
                      (!dy || aligned(dy, 16)) && (!ds || aligned(ds, 16)) &&
                      (!ddelta || aligned(ddelta, 16));
  if (!vec_ok || (dh_q && (!aligned(dh_q, 16) || !aligned(a16_q, 16))) ||
      (dh_v && (!aligned(dh_v, 16) || !aligned(a16_v, 16))) || (mask_q && !aligned(mask_q, 8)) ||
      (mask_v && !aligned(mask_v, 8)))
    return set_error(TB_EALIGN, "add_rmsnorm_bwd_lora: misaligned buffer");
  // the thread -> chunk mapping tb_add_rmsnorm_bwd plans before it weighs the row count (its
  // reduction order): one chunk of 8 per thread up to 256 threads, else two; rows are batched
  // per CTA here instead of adding chunks
  const int64_t chunks = hidden / 8;
  if (hidden % 8 != 0 || chunks > 512)
    return set_error(TB_EINVAL,
                     "add_rmsnorm_bwd_lora: hidden %lld (takes a multiple of 8 up to 4096; "
                     "tb_lora_dropout_grad_expand + tb_add_rmsnorm_bwd cover the rest)",
                     (long long)hidden);
  const int nch = chunks <= 256 ? 1 : 2;
  const int threads = (int)(((chunks + nch - 1) / nch + 31) / 32 * 32);
  RmsLoraArgs a{s, rstd, weight, dy, pad_idx, ds, dx, ddelta,
                {{dh_q, a16_q, mask_q, scale_q}, {dh_v, a16_v, mask_v, scale_v}}, rows, hidden};
  cudaStream_t st = as_stream(stream);
  if (nch == 2) return launch_rms_lora<2, 1>(a, threads, st);
  if (chunks <= kRowsMaxChunks) return launch_rms_lora_rows(a, st);
  return launch_rms_lora<1, 1>(a, threads, st);
}
