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
  pdl_wait();
  pdl_release();
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
  pdl_wait();
  pdl_release();
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
  pdl_wait();
  pdl_release();
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
  pdl_wait();
  pdl_release();
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

// ---- dropout backward with the rank-16 expansion folded in -----------------------------------
// dx = fp16(dh . fp16(A)) of each adapter (the lora_A input gradient, an fp16 GEMM output under
// autocast, K = 16) is computed where the dropout backward needs it instead of being written by
// two GEMMs and read back: per padded slot p with token tok and column c,
//   grad[p, c] = drop_q'(dx_q[tok, c]) + drop_v'(dx_v[tok, c])      (0 for padding slots)
// with drop'(g) = mask ? g * scale : 0 (g when the adapter has no dropout), each product and the
// sum rounded on their own as in tb_lora_dropout_grad. A CTA holds a 256-column slice of both
// fp16(A) in shared memory; each warp takes rows, lane l its 8 columns of the slice, the
// sixteen products of a column summed in rank order in fp32.
constexpr int kExpandCols = 256;
constexpr int kExpandRowsPerWarp = 2;

__global__ void __launch_bounds__(kThreads)
    lora_dropout_grad_expand(const uint16_t *__restrict__ dhq, const uint16_t *__restrict__ aq,
                             const uint16_t *__restrict__ dhv, const uint16_t *__restrict__ av,
                             const uint8_t *__restrict__ mq, const uint8_t *__restrict__ mv,
                             const int32_t *__restrict__ slot_tok, float *__restrict__ g,
                             int64_t slots, int hidden, float sq, float sv) {
  pdl_wait();
  pdl_release();
  __shared__ uint4 a_sh[2][16][kExpandCols / 8];  // fp16(A) slices: [adapter][rank][8 cols]
  const int c0 = blockIdx.x * kExpandCols;
  const int ncols = min(kExpandCols, hidden - c0);
  for (int e = threadIdx.x; e < 2 * 16 * (kExpandCols / 8); e += blockDim.x) {
    const int ad = e / (16 * (kExpandCols / 8)), rem = e % (16 * (kExpandCols / 8));
    const int r = rem / (kExpandCols / 8), v = rem % (kExpandCols / 8);
    const uint16_t *a = ad == 0 ? aq : av;
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (a != nullptr && v * 8 < ncols)
      val = __ldg(reinterpret_cast<const uint4 *>(a + (int64_t)r * hidden + c0 + v * 8));
    a_sh[ad][r][v] = val;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = c0 + lane * 8;
  const bool live = lane * 8 < ncols;
  const int64_t p0 = ((int64_t)blockIdx.y * (blockDim.x >> 5) + warp) * kExpandRowsPerWarp;
  // every row's slot lookup, dh rows and mask bytes are loaded before the math
  int64_t tok[kExpandRowsPerWarp];
#pragma unroll
  for (int i = 0; i < kExpandRowsPerWarp; ++i)
    tok[i] = p0 + i < slots ? __ldg(slot_tok + p0 + i) : -1;
  uint4 hv4[kExpandRowsPerWarp][2][2];  // [row][adapter][half of the 16 dh values]
  uint2 mk[kExpandRowsPerWarp][2];
#pragma unroll
  for (int i = 0; i < kExpandRowsPerWarp; ++i)
#pragma unroll
    for (int ad = 0; ad < 2; ++ad) {
      const uint16_t *dh = ad == 0 ? dhq : dhv;
      const uint8_t *m = ad == 0 ? mq : mv;
      hv4[i][ad][0] = hv4[i][ad][1] = make_uint4(0u, 0u, 0u, 0u);
      mk[i][ad] = make_uint2(0x01010101u, 0x01010101u);
      if (tok[i] >= 0 && live && dh != nullptr) {
        hv4[i][ad][0] = __ldg(reinterpret_cast<const uint4 *>(dh + tok[i] * 16));
        hv4[i][ad][1] = __ldg(reinterpret_cast<const uint4 *>(dh + tok[i] * 16 + 8));
        if (m != nullptr)
          mk[i][ad] = __ldg(reinterpret_cast<const uint2 *>(m + (p0 + i) * hidden + c));
      }
    }
#pragma unroll
  for (int i = 0; i < kExpandRowsPerWarp; ++i) {
    const int64_t p = p0 + i;
    if (p >= slots || !live) continue;
    float out[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) out[k] = 0.f;
    if (tok[i] >= 0) {
#pragma unroll
      for (int ad = 0; ad < 2; ++ad) {
        const uint16_t *dh = ad == 0 ? dhq : dhv;
        if (dh == nullptr) continue;
        const uint8_t *m = ad == 0 ? mq : mv;
        const float scale = ad == 0 ? sq : sv;
        float hf[16];
        const uint32_t hw[8] = {hv4[i][ad][0].x, hv4[i][ad][0].y, hv4[i][ad][0].z, hv4[i][ad][0].w,
                                hv4[i][ad][1].x, hv4[i][ad][1].y, hv4[i][ad][1].z, hv4[i][ad][1].w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float2 f = unpack_half2(hw[j]);
          hf[2 * j] = f.x;
          hf[2 * j + 1] = f.y;
        }
        float acc[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] = 0.f;
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          const uint4 av4 = a_sh[ad][r][lane];
          const uint32_t aw[4] = {av4.x, av4.y, av4.z, av4.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = unpack_half2(aw[j]);
            acc[2 * j] = fmaf(hf[r], f.x, acc[2 * j]);
            acc[2 * j + 1] = fmaf(hf[r], f.y, acc[2 * j + 1]);
          }
        }
        const uint8_t *mb = reinterpret_cast<const uint8_t *>(&mk[i][ad]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float dx = __half2float(__float2half_rn(acc[k]));  // the fp16 GEMM output
          const float gk = m == nullptr ? dx : (mb[k] ? __fmul_rn(dx, scale) : 0.f);
          out[k] = ad == 0 ? gk : __fadd_rn(out[k], gk);
        }
      }
    }
    store8f(g + p * hidden + c, out);
  }
}

// ---- the adapters' forward in one kernel (rank 16) -------------------------------------------
// Per tile of 16 real rows and adapter (blockIdx.y: 0 = q, 1 = v):
//   x16 = fp16(dropped[pos_idx[m]])                         (index_select + the autocast cast)
//   h16 = fp16(x16 . fp16(A)^T)                               (lora_A, fp16 GEMM output)
//   out = fp16(fp32(fp16(h16 . fp16(B)^T)) * scaling)          (lora_B, then * scaling)
// on the tensor cores (mma.sync m16n8k16, fp16 inputs, fp32 accumulation). A thread-block
// cluster of kCluster CTAs takes one tile: CTA r of the cluster takes the r-th 1/kCluster of
// lora_A's K (hidden), its 8 warps split those k-steps and add their partial 16x16 sums in
// shared memory in a fixed order; the cluster then adds the CTAs' sums through distributed
// shared memory, in rank order in every CTA (the same h16 everywhere, deterministic), and CTA r
// computes the r-th interleaved share of lora_B's 16x8 output tiles with h16 as the A operand.
// So a tile's serial chain is 1/kCluster of K and of the output columns, and 621 rows give
// 39 x 2 clusters = 624 CTAs (one wave) instead of 78 CTAs that each walk all of K. Operands
// are read straight from global memory (the weights are L2-resident after the first tiles) and
// rounded to fp16 in registers, so the autocast casts cost no kernel of their own; the cluster
// of tile 0 writes those fp16 weights, and every CTA its share of x16 (h16: rank 0), for the
// backward GEMMs.
constexpr int kRank = 16;
constexpr int kFwdWarps = 8;
constexpr int kCluster = 8;
constexpr int kTileRows = 32;  // rows per cluster: two m16 tiles sharing every A fragment
constexpr int kBPre = 3;       // lora_B output tiles per warp whose operands are loaded early

struct LoraFwdAdapter {
  const float *dropped;  // fp32 [slots, hidden]
  const float *a;        // lora_A weight fp32 [16, hidden]
  const float *b;        // lora_B weight fp32 [hout, 16]
  uint16_t *a16;         // fp16(a), written by tile 0
  uint16_t *b16;         // fp16(b), written by tile 0
  uint16_t *x16;         // fp16 [rows, hidden]
  uint16_t *h16;         // fp16 [rows, 16]
  uint16_t *out;         // fp16 [rows, hout]
  int hout;
  float scale;
};

struct LoraFwdArgs {
  LoraFwdAdapter ad[2];
  const int64_t *pos_idx;
  int64_t rows;
  int hidden;
};

__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// two consecutive fp32 values as one fp16x2 (lower address in the lower half)
__device__ __forceinline__ uint32_t ld_f16x2(const float *p) {
  const float2 v = __ldg(reinterpret_cast<const float2 *>(p));
  return pack_half2(v.x, v.y);
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// every thread of every CTA of the cluster; release/acquire orders shared-memory writes before
// the barrier with reads (local or remote) after it
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

// a float of CTA `rank`'s shared memory at the address `p` has in this CTA
__device__ __forceinline__ float ld_cluster(const float *p, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(p)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// lora_A's work for one k-step of 16 columns: the fp16 x fragments of both 16-row m-tiles
// (rows m0 + 16 mt + g, + 8), the fp16 A fragments of both 8-rank n-tiles, four mma
struct KStep {
  uint32_t x[2][4];  // [m-tile][a0..a3]
  uint32_t w[4];     // b00, b01, b10, b11
};

__device__ __forceinline__ void lora_a_step(const float *const (&xr)[2][2], const float *A, int H,
                                            int k, float (&c)[2][2][4], KStep &st) {
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    st.x[mt][0] = xr[mt][0] ? ld_f16x2(xr[mt][0] + k) : 0u;
    st.x[mt][1] = xr[mt][1] ? ld_f16x2(xr[mt][1] + k) : 0u;
    st.x[mt][2] = xr[mt][0] ? ld_f16x2(xr[mt][0] + k + 8) : 0u;
    st.x[mt][3] = xr[mt][1] ? ld_f16x2(xr[mt][1] + k + 8) : 0u;
  }
  const int g = (threadIdx.x & 31) >> 2;
  // B = A^T: column n of B is row n of A; n-tile 0 = ranks 0..7, n-tile 1 = 8..15
  st.w[0] = ld_f16x2(A + (int64_t)g * H + k);
  st.w[1] = ld_f16x2(A + (int64_t)g * H + k + 8);
  st.w[2] = ld_f16x2(A + (int64_t)(g + 8) * H + k);
  st.w[3] = ld_f16x2(A + (int64_t)(g + 8) * H + k + 8);
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    mma_16816(c[mt][0], st.x[mt][0], st.x[mt][1], st.x[mt][2], st.x[mt][3], st.w[0], st.w[1]);
    mma_16816(c[mt][1], st.x[mt][0], st.x[mt][1], st.x[mt][2], st.x[mt][3], st.w[2], st.w[3]);
  }
}

// x16 of one k-step's valid rows for the backward
__device__ __forceinline__ void lora_x16_store(const LoraFwdAdapter &p, const bool (&rv)[2][2],
                                               int64_t m0, int H, int k, const KStep &st) {
  const int g = (threadIdx.x & 31) >> 2;
  uint32_t *x16 = reinterpret_cast<uint32_t *>(p.x16);
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    const int64_t r = m0 + 16 * mt + g;
    if (rv[mt][0]) {
      x16[(r * H + k) / 2] = st.x[mt][0];
      x16[(r * H + k + 8) / 2] = st.x[mt][2];
    }
    if (rv[mt][1]) {
      x16[((r + 8) * H + k) / 2] = st.x[mt][1];
      x16[((r + 8) * H + k + 8) / 2] = st.x[mt][3];
    }
  }
}

__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kFwdWarps * 32, 3)
    lora_fwd_kernel(const __grid_constant__ LoraFwdArgs a) {
  pdl_wait();
  pdl_release();
  __shared__ float part[kFwdWarps][kTileRows][kRank + 1];
  __shared__ float cta_sum[kTileRows][kRank];      // this CTA's share of x . A^T (cluster-read)
  __shared__ uint32_t h_sh[kTileRows][kRank / 2];  // h16 of the tile, fp16x2 pairs
  const LoraFwdAdapter &p = a.ad[blockIdx.y];
  if (p.a == nullptr) return;  // the whole cluster (one blockIdx.y)
  const uint32_t rank = cluster_ctarank();
  const int H = a.hidden, HO = p.hout;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;  // mma fragment row group / column pair
  const int64_t tile = blockIdx.x / kCluster;
  const bool writer = tile == 0;
  const int64_t m0 = tile * kTileRows;
  bool rv[2][2];
  const float *xr[2][2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int64_t r = m0 + 16 * mt + 8 * hf + g;
      rv[mt][hf] = r < a.rows;
      xr[mt][hf] = rv[mt][hf] ? p.dropped + __ldg(a.pos_idx + r) * H : nullptr;
    }
  // lora_B's operand fragments of this warp's first kBPre output tiles, loaded now (they do
  // not depend on h): n-tile nt goes to CTA nt % kCluster, within it to warp nt / kCluster %
  // kFwdWarps
  const int nt0 = (int)rank + kCluster * warp;
  constexpr int kStride = kCluster * kFwdWarps;
  uint32_t bpre[kBPre][2];
#pragma unroll
  for (int i = 0; i < kBPre; ++i) {
    const int nt = nt0 + i * kStride;
    if (nt < HO / 8) {
      const int n = nt * 8 + g;  // B[k][n] = lora_B[n][k]
      bpre[i][0] = ld_f16x2(p.b + (int64_t)n * kRank + 2 * t);
      bpre[i][1] = ld_f16x2(p.b + (int64_t)n * kRank + 2 * t + 8);
    }
  }

  // lora_A: this CTA's k-steps of 16 columns over its warps. Nothing is stored to global
  // memory before the cluster barriers (a barrier's release would wait for it): the x16 copies
  // of a warp's first two k-steps wait in registers; further k-steps (hidden > 2048) store as
  // they go.
  float c[2][2][4] = {};
  const int ksteps = H / 16;
  const int kper = (ksteps + kCluster - 1) / kCluster;
  const int kbeg = (int)rank * kper, kend = min(ksteps, kbeg + kper);
  const int ks0 = kbeg + warp, ks1 = ks0 + kFwdWarps;
  KStep s0, s1;
  if (ks0 < kend) lora_a_step(xr, p.a, H, ks0 * 16 + 2 * t, c, s0);
  if (ks1 < kend) lora_a_step(xr, p.a, H, ks1 * 16 + 2 * t, c, s1);
  for (int ks = ks1 + kFwdWarps; ks < kend; ks += kFwdWarps) {
    KStep st;
    lora_a_step(xr, p.a, H, ks * 16 + 2 * t, c, st);
    lora_x16_store(p, rv, m0, H, ks * 16 + 2 * t, st);
  }
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      part[warp][16 * mt + g][8 * nt + 2 * t] = c[mt][nt][0];
      part[warp][16 * mt + g][8 * nt + 2 * t + 1] = c[mt][nt][1];
      part[warp][16 * mt + g + 8][8 * nt + 2 * t] = c[mt][nt][2];
      part[warp][16 * mt + g + 8][8 * nt + 2 * t + 1] = c[mt][nt][3];
    }
  __syncthreads();
  for (int e = threadIdx.x; e < kTileRows * kRank; e += kFwdWarps * 32) {
    // the CTA's 32 x 16 sum, warps added in order
    const int row = e / kRank, col = e % kRank;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kFwdWarps; ++w) s += part[w][row][col];
    cta_sum[row][col] = s;
  }
  cluster_sync();  // every CTA's sum is written
  uint32_t hv = 0;
  const int hrow = threadIdx.x / (kRank / 2), hpr = threadIdx.x % (kRank / 2);
  if (threadIdx.x < kTileRows * kRank / 2) {  // one fp16x2 pair of h each
    float h0 = 0.f, h1 = 0.f;
#pragma unroll
    for (uint32_t r = 0; r < (uint32_t)kCluster; ++r) {  // rank order: the same h16 everywhere
      h0 += ld_cluster(&cta_sum[hrow][2 * hpr], r);
      h1 += ld_cluster(&cta_sum[hrow][2 * hpr + 1], r);
    }
    hv = pack_half2(h0, h1);
    h_sh[hrow][hpr] = hv;
  }
  cluster_sync();  // no CTA leaves while another reads its sums; h_sh complete

  // lora_B: A operand = h16 (two 16 x 16 m-tiles), one 16 x 8 output tile per mma
  uint32_t ha[2][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    ha[mt][0] = h_sh[16 * mt + g][t];
    ha[mt][1] = h_sh[16 * mt + g + 8][t];
    ha[mt][2] = h_sh[16 * mt + g][4 + t];
    ha[mt][3] = h_sh[16 * mt + g + 8][4 + t];
  }
  for (int i = 0, nt = nt0; nt < HO / 8; ++i, nt += kStride) {
    const int n = nt * 8 + g;
    uint32_t b0, b1;
    if (i < kBPre) {
#pragma unroll
      for (int j = 0; j < kBPre; ++j)
        if (j == i) {
          b0 = bpre[j][0];
          b1 = bpre[j][1];
        }
    } else {
      b0 = ld_f16x2(p.b + (int64_t)n * kRank + 2 * t);
      b1 = ld_f16x2(p.b + (int64_t)n * kRank + 2 * t + 8);
    }
    if (writer) {
      uint32_t *w = reinterpret_cast<uint32_t *>(p.b16);
      w[((int64_t)n * kRank + 2 * t) / 2] = b0;
      w[((int64_t)n * kRank + 2 * t + 8) / 2] = b1;
    }
    const int col = nt * 8 + 2 * t;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      float o[4] = {0.f, 0.f, 0.f, 0.f};
      mma_16816(o, ha[mt][0], ha[mt][1], ha[mt][2], ha[mt][3], b0, b1);
      // the GEMM's fp16 output, then * scaling, rounded to fp16 again
      const int64_t r = m0 + 16 * mt + g;
      if (rv[mt][0]) {
        const float2 v = unpack_half2(pack_half2(o[0], o[1]));
        reinterpret_cast<uint32_t *>(p.out)[(r * HO + col) / 2] =
            pack_half2(v.x * p.scale, v.y * p.scale);
      }
      if (rv[mt][1]) {
        const float2 v = unpack_half2(pack_half2(o[2], o[3]));
        reinterpret_cast<uint32_t *>(p.out)[((r + 8) * HO + col) / 2] =
            pack_half2(v.x * p.scale, v.y * p.scale);
      }
    }
  }
  // the copies for the backward
  if (rank == 0 && threadIdx.x < kTileRows * kRank / 2 && m0 + hrow < a.rows)
    reinterpret_cast<uint32_t *>(p.h16)[(m0 + hrow) * (kRank / 2) + hpr] = hv;
  if (ks0 < kend) lora_x16_store(p, rv, m0, H, ks0 * 16 + 2 * t, s0);
  if (ks1 < kend) lora_x16_store(p, rv, m0, H, ks1 * 16 + 2 * t, s1);
  if (writer) {  // fp16(A) of this CTA's k-range (re-read: L2-resident)
    uint32_t *w = reinterpret_cast<uint32_t *>(p.a16);
    const int k0 = kbeg * 16, k1 = kend * 16;
    for (int e = threadIdx.x; e < kRank * (k1 - k0) / 2; e += kFwdWarps * 32) {
      const int row = e / ((k1 - k0) / 2), k = k0 + 2 * (e % ((k1 - k0) / 2));
      w[((int64_t)row * H + k) / 2] = ld_f16x2(p.a + (int64_t)row * H + k);
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
    return launch("lora_gather", lora_gather_vec, grid_for(rows * hidden / 8), kThreads, 0, st,
                  dropped_q, dropped_v, pos_idx, xq, xv, rows, hidden / 8);
  }
  return launch("lora_gather", lora_gather_any, grid_for(rows * hidden), kThreads, 0, st,
                dropped_q, dropped_v, pos_idx, xq, xv, rows, hidden);
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
    return launch("lora_dropout_grad", lora_dropout_grad_vec, grid_for(slots * hidden / 8),
                  kThreads, 0, st, dxq, dxv, mask_q, mask_v, slot_tok, grad, slots, hidden / 8,
                  scale_q, scale_v);
  }
  return launch("lora_dropout_grad", lora_dropout_grad_any, grid_for(slots * hidden), kThreads, 0,
                st, dxq, dxv, mask_q, mask_v, slot_tok, grad, slots, hidden, scale_q, scale_v);
}

extern "C" int tb_lora_dropout_grad_expand(const uint16_t *dh_q, const uint16_t *a16_q,
                                           const uint16_t *dh_v, const uint16_t *a16_v,
                                           const uint8_t *mask_q, const uint8_t *mask_v,
                                           const int32_t *slot_tok, float *grad, int64_t slots,
                                           int64_t hidden, int32_t rank, float scale_q,
                                           float scale_v, void *stream) {
  if (rank != 16)
    return set_error(TB_EINVAL, "lora_dropout_grad_expand: rank %d (the kernel takes rank 16)",
                     rank);
  if (slots < 0 || hidden <= 0 || hidden % 8 || hidden > (1 << 30))
    return set_error(TB_EINVAL, "lora_dropout_grad_expand: slots %lld hidden %lld",
                     (long long)slots, (long long)hidden);
  if (slots == 0) return TB_OK;
  if (!slot_tok || !grad) return set_error(TB_EINVAL, "lora_dropout_grad_expand: slot_tok, grad required");
  if ((dh_q && !a16_q) || (dh_v && !a16_v))
    return set_error(TB_EINVAL, "lora_dropout_grad_expand: an adapter's dh needs its fp16 A");
  if (!aligned(grad, 16) || (dh_q && (!aligned(dh_q, 16) || !aligned(a16_q, 16))) ||
      (dh_v && (!aligned(dh_v, 16) || !aligned(a16_v, 16))) || (mask_q && !aligned(mask_q, 8)) ||
      (mask_v && !aligned(mask_v, 8)))
    return set_error(TB_EALIGN, "lora_dropout_grad_expand: misaligned buffer");
  const int64_t rows_per_cta = (int64_t)(kThreads / 32) * kExpandRowsPerWarp;
  const int64_t ys = (slots + rows_per_cta - 1) / rows_per_cta;
  if (ys > 65535) return set_error(TB_EINVAL, "lora_dropout_grad_expand: too many slots");
  const dim3 grid((unsigned)((hidden + kExpandCols - 1) / kExpandCols), (unsigned)ys);
  return launch("lora_dropout_grad_expand", lora_dropout_grad_expand, grid, kThreads, 0,
                as_stream(stream), dh_q, a16_q, dh_v, a16_v, mask_q, mask_v, slot_tok, grad, slots,
                (int)hidden, scale_q, scale_v);
}

extern "C" int tb_lora_forward(const float *dropped_q, const float *a_q, const float *b_q,
                               uint16_t *a16_q, uint16_t *b16_q, uint16_t *x16_q,
                               uint16_t *h16_q, uint16_t *out_q, int64_t hout_q, float scale_q,
                               const float *dropped_v, const float *a_v, const float *b_v,
                               uint16_t *a16_v, uint16_t *b16_v, uint16_t *x16_v,
                               uint16_t *h16_v, uint16_t *out_v, int64_t hout_v, float scale_v,
                               const int64_t *pos_idx, int64_t rows, int64_t hidden, int32_t rank,
                               void *stream) {
  if (rank != kRank)
    return set_error(TB_EINVAL, "lora_forward: rank %d (the fused kernel takes rank %d)", rank,
                     kRank);
  if (rows < 0 || hidden <= 0 || hidden % 16 || hout_q % 8 || hout_v % 8 || hout_q < 0 ||
      hout_v < 0)
    return set_error(TB_EINVAL, "lora_forward: rows %lld hidden %lld hout %lld/%lld",
                     (long long)rows, (long long)hidden, (long long)hout_q, (long long)hout_v);
  if (!a_q && !a_v) return TB_OK;
  if (rows > (1LL << 31) / (hidden > 16 ? hidden : 16))
    return set_error(TB_EINVAL, "lora_forward: too many rows");
  LoraFwdArgs args{};
  const float *dr[2] = {dropped_q, dropped_v}, *aa[2] = {a_q, a_v}, *bb[2] = {b_q, b_v};
  uint16_t *a16[2] = {a16_q, a16_v}, *b16[2] = {b16_q, b16_v};
  uint16_t *xx[2] = {x16_q, x16_v}, *hh[2] = {h16_q, h16_v}, *oo[2] = {out_q, out_v};
  const int64_t ho[2] = {hout_q, hout_v};
  const float sc[2] = {scale_q, scale_v};
  for (int i = 0; i < 2; ++i) {
    if (aa[i] == nullptr) continue;
    if (!bb[i] || !a16[i] || !b16[i] || (rows > 0 && (!dr[i] || !xx[i] || !hh[i] || !oo[i])))
      return set_error(TB_EINVAL,
                       "lora_forward: adapter %d needs dropped, a, b, a16, b16, x16, h16, out", i);
    if (!aligned(aa[i], 8) || !aligned(bb[i], 8) || !aligned(a16[i], 4) || !aligned(b16[i], 4) ||
        (rows > 0 && (!aligned(dr[i], 8) || !aligned(xx[i], 4) || !aligned(hh[i], 4) ||
                      !aligned(oo[i], 4))))
      return set_error(TB_EALIGN, "lora_forward: misaligned buffer");
    args.ad[i] = LoraFwdAdapter{dr[i], aa[i], bb[i], a16[i], b16[i], xx[i], hh[i], oo[i],
                                (int)ho[i], sc[i]};
  }
  if (rows > 0 && !pos_idx) return set_error(TB_EINVAL, "lora_forward: pos_idx is required");
  args.pos_idx = pos_idx;
  args.rows = rows;
  args.hidden = (int)hidden;
  // one cluster of kCluster CTAs per kTileRows rows and adapter (tile 0 also writes the fp16
  // weights, so at least one)
  const int64_t tiles = rows > 0 ? (rows + kTileRows - 1) / kTileRows : 1;
  if (tiles * kCluster > 0x7fffffffLL) return set_error(TB_EINVAL, "lora_forward: too many rows");
  return launch("lora_forward", lora_fwd_kernel, dim3((unsigned)(tiles * kCluster), 2),
                kFwdWarps * 32, 0, as_stream(stream), args);
}
