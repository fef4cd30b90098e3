// The rank-16 LoRA backward of both adapters (q_proj and v_proj) of a layer in two launches,
// in place of six cuBLAS GEMMs (reference: peft's lora_B(lora_A(dropout(x))) * scaling under
// fp16 autocast, solution/model.py:195-206; its backward as the LoRA pair node computes it):
//
//   per adapter, g = d(out) fp16 [M, W], h = lora_A output fp16 [M, 16], B16 = fp16(lora_B)
//   [W, 16], x16 = fp16 lora_A input [M, H], s = scaling:
//     dh = fp16(s * g . B16)            [M, 16]   (kernel 1, a CTA per 16 rows, both adapters)
//     dB = s * g^T . h  (+ dB)          [W, 16]   fp32 (kernel 1, a CTA per 64 output features)
//     dA = dh^T . x16   (+ dA)          [16, H]   fp32 (kernel 2, a CTA per 64 input features)
// "(+ ...)" when the gradient is accumulated in place (a gradient bucket's view), as the GEMMs
// with beta 1 do. The lora_A input gradient dh . fp16(A) stays in tb_lora_dropout_grad_expand.
//
// Every product is mma.sync m16n8k16 (fp16 operands, fp32 accumulation). The eight warps of a
// CTA take alternate 16-wide chunks of the reduction; each warp stages its chunks' operands
// through its own double-buffered shared memory (cp.async, zero-filled past the last row) and
// reads them with ldmatrix (.trans where the reduction runs along the rows of both operands);
// the warps' partial sums are added in warp order, so every result is deterministic.
#include "common.cuh"

namespace tb {
namespace {

constexpr int kRank = 16;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kCols = 64;            // output columns of a dB / dA CTA
constexpr int kLdP = kRank + 8;      // 48-byte rows: conflict-free ldmatrix
constexpr int kLdQ = kCols + 8;      // 144-byte rows
constexpr int kPHalves = 16 * kLdP;
constexpr int kQHalves = 16 * kLdQ;
constexpr int kWarpHalves = 2 * (kPHalves + kQHalves);  // two buffers
constexpr int kSmemBytes = kWarps * kWarpHalves * 2;    // 48 KB
static_assert(kWarps * 16 * kCols * 4 <= kSmemBytes, "the reduction reuses the staging buffers");

struct Adapter {
  const uint16_t *g;    // fp16 [M, W], row stride ld_g
  const uint16_t *h;    // fp16 [M, 16]
  const uint16_t *b16;  // fp16 [W, 16]
  const uint16_t *x16;  // fp16 [M, H]
  uint16_t *dh;         // fp16 [M, 16] out
  float *db;            // fp32 [W, 16]
  float *da;            // fp32 [16, H]
  int width;            // W
  int64_t ld_g;         // row stride of g (>= W)
  float scale;
  bool acc_db, acc_da;
};

struct BwdArgs {
  Adapter ad[2];
  int rows;     // M
  int hidden;   // H
  int m_tiles;  // ceil(M / 16): the dh CTAs of kernel 1
  int nb[2];    // W / 64 per adapter (0 when absent): the dB CTAs of kernel 1
  int hb[2];    // H / 64 per present adapter: the CTAs of kernel 2
};

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm4_t(uint32_t (&r)[4], const uint16_t *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// 16 bytes global -> shared, asynchronously; zero-filled when !in (src then unused)
__device__ __forceinline__ void cp16(uint16_t *dst, const uint16_t *src, bool in) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(in ? 16 : 0)
               : "memory");
}

__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t ld_u32(const uint16_t *p) {
  return __ldg(reinterpret_cast<const unsigned int *>(p));
}

// ---- dh = fp16(s * g . B16) for rows m0 .. m0 + 15 ----------------------------------------
// C[m, r] over chunks of 16 of W: A = g rows (fragments straight from global memory, the next
// chunk's loaded before the current chunk's MMAs), B = B16 rows n0 .. n0 + 15 staged in shared
// memory and read with ldmatrix.trans (B[k = n][r] is a row-major [n, r] block).
__device__ void dh_rows(const Adapter &ad, int rows, int m0, uint16_t *wbuf, float *red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int chunks = ad.width >> 4;
  const bool r0_in = m0 + g < rows, r1_in = m0 + g + 8 < rows;
  const uint16_t *g0 = ad.g + (int64_t)(r0_in ? m0 + g : 0) * ad.ld_g + 2 * t;
  const uint16_t *g1 = ad.g + (int64_t)(r1_in ? m0 + g + 8 : 0) * ad.ld_g + 2 * t;
  float c[2][4] = {};
  auto stage = [&](int kc, int b) {  // 16 rows x 32 bytes: one 16-byte copy per lane
    const int r = lane >> 1, col = (lane & 1) * 8;
    cp16(wbuf + b * kPHalves + r * kLdP + col, ad.b16 + (int64_t)(kc * 16 + r) * kRank + col, true);
    cp_commit();
  };
  auto afrag = [&](int kc, uint32_t (&a)[4]) {
    const int n0 = kc * 16;
    a[0] = r0_in ? ld_u32(g0 + n0) : 0u;
    a[1] = r1_in ? ld_u32(g1 + n0) : 0u;
    a[2] = r0_in ? ld_u32(g0 + n0 + 8) : 0u;
    a[3] = r1_in ? ld_u32(g1 + n0 + 8) : 0u;
  };
  int buf = 0;
  uint32_t a[4] = {0u, 0u, 0u, 0u};
  if (warp < chunks) {
    stage(warp, 0);
    afrag(warp, a);
  }
  for (int kc = warp; kc < chunks; kc += kWarps) {
    const int nk = kc + kWarps;
    uint32_t an[4] = {0u, 0u, 0u, 0u};
    if (nk < chunks) {
      stage(nk, buf ^ 1);
      afrag(nk, an);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncwarp();
    // matrices: (n 0-7, r 0-7) (n 8-15, r 0-7) (n 0-7, r 8-15) (n 8-15, r 8-15)
    const int q = lane >> 3, i = lane & 7;
    uint32_t b[4];
    ldsm4_t(b, wbuf + buf * kPHalves + (i + (q & 1) * 8) * kLdP + (q >> 1) * 8);
    mma16816(c[0], a, b[0], b[1]);
    mma16816(c[1], a, b[2], b[3]);
    __syncwarp();
#pragma unroll
    for (int e = 0; e < 4; ++e) a[e] = an[e];
    buf ^= 1;
  }
  // red[warp][m][r]
  float *mine = red + warp * 256;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    mine[g * 16 + 8 * j + 2 * t] = c[j][0];
    mine[g * 16 + 8 * j + 2 * t + 1] = c[j][1];
    mine[(g + 8) * 16 + 8 * j + 2 * t] = c[j][2];
    mine[(g + 8) * 16 + 8 * j + 2 * t + 1] = c[j][3];
  }
  __syncthreads();
  const int m = threadIdx.x >> 4, r = threadIdx.x & 15;  // 256 threads: one (m, r) each
  float sum = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) sum = __fadd_rn(sum, red[w * 256 + m * 16 + r]);
  if (m0 + m < rows)
    ad.dh[(int64_t)(m0 + m) * kRank + r] = __half_as_ushort(__float2half_rn(__fmul_rn(sum, ad.scale)));
  __syncthreads();  // red is reused by the next adapter
}

// ---- C[r, n] = sum_m P[m, r] Q[m, n0 + n] over all rows, n < 64 --------------------------------
// P fp16 [M, 16] (h or dh), Q fp16 [M, ldq] (g or x16). Both operands have the reduction along
// their rows: 16-row chunks staged per warp, A = P^T and B = Q by ldmatrix.trans. Result (times
// `scale`, plus the old value when `acc`) to out[n * 16 + r] (transposed: dB [W, 16]) or
// out[r * ldo + n] (dA [16, H]).
__device__ void tn_cols(const uint16_t *P, const uint16_t *Q, int64_t ldq, int rows, int n0,
                        float scale, float *out, int64_t ldo, bool transposed, bool acc,
                        uint16_t *smem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  uint16_t *wbuf = smem + warp * kWarpHalves;
  const int chunks = (rows + 15) >> 4;
  float c[8][4] = {};
  auto stage = [&](int kc, int b) {
    const int m0 = kc * 16;
    uint16_t *ps = wbuf + b * (kPHalves + kQHalves);
    uint16_t *qs = ps + kPHalves;
    {
      const int r = lane >> 1, col = (lane & 1) * 8;
      const bool in = m0 + r < rows;
      cp16(ps + r * kLdP + col, in ? P + (int64_t)(m0 + r) * kRank + col : P, in);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int e = lane + 32 * k, r = e >> 3, col = (e & 7) * 8;
      const bool in = m0 + r < rows;
      cp16(qs + r * kLdQ + col, in ? Q + (int64_t)(m0 + r) * ldq + n0 + col : Q, in);
    }
    cp_commit();
  };
  int buf = 0;
  if (warp < chunks) stage(warp, 0);
  for (int kc = warp; kc < chunks; kc += kWarps) {
    const int nk = kc + kWarps;
    if (nk < chunks) {
      stage(nk, buf ^ 1);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncwarp();
    const uint16_t *ps = wbuf + buf * (kPHalves + kQHalves);
    const uint16_t *qs = ps + kPHalves;
    const int q = lane >> 3, i = lane & 7;
    // A = P^T: a0..a3 from the P blocks (m 0-7, r 0-7) (m 0-7, r 8-15) (m 8-15, r 0-7)
    // (m 8-15, r 8-15)
    uint32_t a[4];
    ldsm4_t(a, ps + (i + (q >> 1) * 8) * kLdP + (q & 1) * 8);
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      // B = Q: (m 0-7, n 8j) (m 8-15, n 8j) (m 0-7, n 8j+8) (m 8-15, n 8j+8)
      uint32_t b[4];
      ldsm4_t(b, qs + (i + (q & 1) * 8) * kLdQ + 8 * j + (q >> 1) * 8);
      mma16816(c[j], a, b[0], b[1]);
      mma16816(c[j + 1], a, b[2], b[3]);
    }
    __syncwarp();
    buf ^= 1;
  }
  __syncthreads();  // every warp is done with its staging buffers: reuse them for the sums
  float *red = reinterpret_cast<float *>(smem);
  float *mine = red + warp * (16 * kCols);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    mine[g * kCols + 8 * j + 2 * t] = c[j][0];
    mine[g * kCols + 8 * j + 2 * t + 1] = c[j][1];
    mine[(g + 8) * kCols + 8 * j + 2 * t] = c[j][2];
    mine[(g + 8) * kCols + 8 * j + 2 * t + 1] = c[j][3];
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < (16 * kCols) / kThreads; ++k) {
    const int e = threadIdx.x + kThreads * k;
    const int r = e / kCols, n = e % kCols;
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) sum = __fadd_rn(sum, red[w * 16 * kCols + e]);
    float *o = transposed ? out + (int64_t)(n0 + n) * kRank + r : out + (int64_t)r * ldo + n0 + n;
    const float v = __fmul_rn(sum, scale);
    *o = acc ? __fadd_rn(*o, v) : v;
  }
}

// kernel 1: CTAs [0, m_tiles) dh of 16 rows (both adapters); then the dB CTAs of adapter 0, 1
__global__ void __launch_bounds__(kThreads) lora_bwd_dh_db(const __grid_constant__ BwdArgs a) {
  pdl_wait();
  pdl_release();
  extern __shared__ __align__(16) uint16_t smem[];
  int cta = blockIdx.x;
  if (cta < a.m_tiles) {
    const int warp = threadIdx.x >> 5;
    float *red = reinterpret_cast<float *>(smem + kWarps * 2 * kPHalves);
    for (int j = 0; j < 2; ++j)
      if (a.ad[j].g != nullptr)
        dh_rows(a.ad[j], a.rows, cta * 16, smem + warp * 2 * kPHalves, red);
    return;
  }
  cta -= a.m_tiles;
  const int j = cta < a.nb[0] ? 0 : 1;
  const int blk = j == 0 ? cta : cta - a.nb[0];
  const Adapter &ad = a.ad[j];
  tn_cols(ad.h, ad.g, ad.ld_g, a.rows, blk * kCols, ad.scale, ad.db, 0, true, ad.acc_db, smem);
}

// kernel 2: dA of adapter 0 (CTAs [0, hb[0])) and adapter 1
__global__ void __launch_bounds__(kThreads) lora_bwd_da(const __grid_constant__ BwdArgs a) {
  pdl_wait();
  pdl_release();
  extern __shared__ __align__(16) uint16_t smem[];
  const int cta = blockIdx.x;
  const int j = cta < a.hb[0] ? 0 : 1;
  const int blk = j == 0 ? cta : cta - a.hb[0];
  const Adapter &ad = a.ad[j];
  tn_cols(ad.dh, ad.x16, a.hidden, a.rows, blk * kCols, 1.f, ad.da, a.hidden, false, ad.acc_da,
          smem);
}

// One event per device for the fork of kernel 2 onto a second stream (created on first use,
// kept until exit; recording it again, also inside a stream capture, starts a new fork).
cudaEvent_t fork_event() {
  static cudaEvent_t events[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (events[dev] == nullptr &&
      cudaEventCreateWithFlags(&events[dev], cudaEventDisableTiming) != cudaSuccess)
    return nullptr;
  return events[dev];
}

}  // namespace
}  // namespace tb

using namespace tb;

// Per adapter (q, then v; an adapter whose g is NULL is skipped): g, h, b16, x16 inputs,
// dh fp16 output, db / da fp32 outputs (accumulated into when bit 0 / bit 1 of `accumulate`'s
// byte for the adapter is set: bits 0-1 adapter q, bits 2-3 adapter v).
extern "C" int tb_lora_backward(const uint16_t *g_q, const uint16_t *h_q, const uint16_t *b16_q,
                                const uint16_t *x16_q, uint16_t *dh_q, float *db_q, float *da_q,
                                int64_t width_q, float scale_q, const uint16_t *g_v,
                                const uint16_t *h_v, const uint16_t *b16_v, const uint16_t *x16_v,
                                uint16_t *dh_v, float *db_v, float *da_v, int64_t width_v,
                                float scale_v, int64_t rows, int64_t hidden, int32_t rank,
                                int32_t accumulate, int64_t ld_g_q, int64_t ld_g_v,
                                void *stream, void *stream_da) {
  if (rank != kRank) return set_error(TB_EINVAL, "lora_backward: rank %d (the kernels take 16)", rank);
  if (rows < 0 || rows > (1LL << 24) || hidden <= 0 || hidden % kCols != 0 || hidden > (1LL << 20))
    return set_error(TB_EINVAL, "lora_backward: rows %lld hidden %lld (a multiple of %d)",
                     (long long)rows, (long long)hidden, kCols);
  BwdArgs a;
  const uint16_t *gs[2] = {g_q, g_v}, *hs[2] = {h_q, h_v}, *bs[2] = {b16_q, b16_v},
                 *xs[2] = {x16_q, x16_v};
  uint16_t *dhs[2] = {dh_q, dh_v};
  float *dbs[2] = {db_q, db_v}, *das[2] = {da_q, da_v};
  const int64_t widths[2] = {width_q, width_v}, lds[2] = {ld_g_q, ld_g_v};
  const float scales[2] = {scale_q, scale_v};
  for (int j = 0; j < 2; ++j) {
    Adapter &ad = a.ad[j];
    ad = Adapter{};
    a.nb[j] = 0;
    a.hb[j] = 0;
    if (gs[j] == nullptr) continue;
    if (!hs[j] || !bs[j] || !xs[j] || !dhs[j] || !dbs[j] || !das[j])
      return set_error(TB_EINVAL, "lora_backward: adapter %d has a missing buffer", j);
    if (widths[j] <= 0 || widths[j] % kCols != 0 || widths[j] > (1LL << 20))
      return set_error(TB_EINVAL, "lora_backward: adapter %d width %lld (a multiple of %d)", j,
                       (long long)widths[j], kCols);
    if (lds[j] < widths[j] || lds[j] % 8 != 0)
      return set_error(TB_EINVAL, "lora_backward: adapter %d row stride %lld (>= width, 16-byte "
                       "rows)", j, (long long)lds[j]);
    // g, h, B16, x16 and dh (kernel 2 reads it back) go through 16-byte cp.async copies
    if (!aligned(gs[j], 16) || !aligned(hs[j], 16) || !aligned(bs[j], 16) || !aligned(xs[j], 16) ||
        !aligned(dhs[j], 16) || !aligned(dbs[j], 4) || !aligned(das[j], 4))
      return set_error(TB_EALIGN, "lora_backward: adapter %d has a misaligned buffer", j);
    ad.g = gs[j];
    ad.h = hs[j];
    ad.b16 = bs[j];
    ad.x16 = xs[j];
    ad.dh = dhs[j];
    ad.db = dbs[j];
    ad.da = das[j];
    ad.width = (int)widths[j];
    ad.ld_g = lds[j];
    ad.scale = scales[j];
    ad.acc_db = (accumulate >> (2 * j)) & 1;
    ad.acc_da = (accumulate >> (2 * j + 1)) & 1;
    a.nb[j] = (int)(widths[j] / kCols);
    a.hb[j] = (int)(hidden / kCols);
  }
  if (!g_q && !g_v) return TB_OK;
  a.rows = (int)rows;
  a.hidden = (int)hidden;
  a.m_tiles = (int)((rows + 15) / 16);
  // an absent adapter q has empty CTA ranges (nb[0] = hb[0] = 0): every CTA maps to v
  const int grid1 = a.m_tiles + a.nb[0] + a.nb[1];
  const int grid2 = a.hb[0] + a.hb[1];
  int rc = TB_OK;
  if (grid1 > 0)
    rc = launch("lora_bwd_dh_db", lora_bwd_dh_db, dim3((unsigned)grid1), dim3(kThreads),
                (size_t)kSmemBytes, as_stream(stream), a);
  if (rc != TB_OK) return rc;  // with no rows, kernel 2 still writes (or keeps) zero dA
  // kernel 2 on the caller's second stream, after kernel 1 (an event of this library's), so it
  // runs beside whatever the caller queues next on `stream`; the caller joins the two streams
  cudaStream_t st2 = as_stream(stream);
  if (stream_da != nullptr && stream_da != stream) {
    cudaEvent_t ev = fork_event();
    if (ev == nullptr) return set_error(TB_ELAUNCH, "lora_backward: no fork event");
    if (cudaEventRecord(ev, as_stream(stream)) != cudaSuccess ||
        cudaStreamWaitEvent(as_stream(stream_da), ev, 0) != cudaSuccess)
      return check_launch("lora_backward fork");
    st2 = as_stream(stream_da);
  }
  return launch("lora_bwd_da", lora_bwd_da, dim3((unsigned)grid2), dim3(kThreads),
                (size_t)kSmemBytes, st2, a);
}
