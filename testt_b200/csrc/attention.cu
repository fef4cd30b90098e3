// Causal variable-length attention with grouped key/value heads, for sm_100a.
//
// Reference: the attention of the decoder layer (solution/model.py:242-247: SDPA over the padded
// [batch, heads, seq, 128] layout with the causal + padding mask). Here the q/k/v of the real
// tokens are token-major ([tokens, heads, 128], packed sequences given by cu_seqlens), and each
// query attends to the keys of its own sequence up to its own position: the same outputs for
// the real rows, with no padded position computed.
//
// At the step's sizes (4 sequences of 131-193 tokens, 12 query heads over 2 key/value heads,
// head dim 128) the work is small (about 0.3 GFLOP forward per layer) and latency-bound, so the
// kernels are plain tensor-core tiles (mma.sync m16n8k16, fp16 operands, fp32 accumulation)
// staged through shared memory (cp.async, the next block copied while one is used) and read
// with ldmatrix, one CTA per (64-query block, head, sequence), two warp groups per CTA taking
// alternate key (or query) blocks and merging their partial results at the end, so a CTA's
// serial chain is half its blocks. The grid is (heads, sequences, blocks) with the blocks that
// have the most work launched first (the last query block; for dK/dV key block 0), so at one
// CTA per SM the CTAs left for a second wave are the shortest:
//   forward   S = Q K^T, online softmax in base 2 (the scale folded with log2 e), O += P V;
//             writes O (fp16) and the base-2 log-sum-exp per (head, query) for the backward.
// Rows of a sequence's last block past its length are computed but never stored.
#include <math_constants.h>

#include "common.cuh"

namespace tb {
namespace {

constexpr int kD = 128;       // head dimension the kernels take
constexpr int kBlock = 64;    // queries per CTA, keys per step
constexpr int kLd = kD + 8;   // shared-memory row stride in halves (272 B: conflict-free ldmatrix)
constexpr int kWarps = 4;     // per warp group: 16 rows each
constexpr int kCtaThreads = 2 * kWarps * 32;  // two warp groups take alternate blocks
constexpr int kTileHalves = kBlock * kLd;

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// four 8x8 fp16 matrices; lane i gives the row address of matrix i / 8 (row i % 8)
__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], const uint16_t *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm4_t(uint32_t (&r)[4], const uint16_t *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ float attn_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// rows [0, nrows) of a 64 x 128 tile from a token-major tensor (row stride ld halves) into
// shared memory, asynchronously (cp.async, 16 bytes a copy, threads tid of nthr; rows past
// nrows are zero-filled)
__device__ __forceinline__ void load_tile_async(uint16_t *sm, const uint16_t *g, int64_t ld,
                                                int nrows, int tid, int nthr) {
  for (int i = tid; i < kBlock * (kD / 8); i += nthr) {
    const int r = i >> 4, c = (i & 15) * 8;
    const bool in = r < nrows;
    const uint16_t *src = g + (in ? r * ld + c : 0);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(sm + r * kLd + c)),
                 "l"(src), "r"(in ? 16 : 0)
                 : "memory");
  }
}

// barrier of one warp group (4 warps) of the CTA
__device__ __forceinline__ void wg_sync(int wg) {
  asm volatile("bar.sync %0, %1;" ::"r"(wg + 1), "r"(kWarps * 32) : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// A-operand fragments (16 rows starting at r0, 8 chunks of 16 columns) of a 64 x 128 tile
__device__ __forceinline__ void load_a_frags(uint32_t (&a)[8][4], const uint16_t *tile, int r0) {
  const int lane = threadIdx.x & 31;
  const int r = r0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int c = (lane >> 4) * 8;
#pragma unroll
  for (int kc = 0; kc < 8; ++kc) ldsm4(a[kc], tile + r * kLd + kc * 16 + c);
}

struct FwdArgs {
  const uint16_t *q, *k, *v;
  const int32_t *cu;
  uint16_t *out;
  float *lse;  // [n_heads, total] base-2 log-sum-exp of the scaled scores
  int64_t total;
  int n_heads, n_kv;
  float scale_log2;  // softmax scale * log2(e)
};

__global__ void __launch_bounds__(kCtaThreads) attn_fwd_kernel(const __grid_constant__ FwdArgs a) {
  pdl_wait();
  pdl_release();
  extern __shared__ __align__(16) uint16_t smem[];
  // tile 0: Q; warp group w: tiles 1 + 4w .. 4 + 4w, (K, V) twice: its next key block is
  // copied while it uses one. Group w takes key blocks w, w + 2, ...; the two online-softmax
  // states are merged at the end.
  // grid (heads, batch, query blocks), the last query block first: the longest causal blocks
  // start in the first wave and the shortest fill the tail
  const int qb = (int)(gridDim.z - 1 - blockIdx.z), h = blockIdx.x, b = blockIdx.y;
  const int start = __ldg(a.cu + b), len = __ldg(a.cu + b + 1) - start;
  const int q0 = qb * kBlock;
  if (q0 >= len) return;
  const int hk = h / (a.n_heads / a.n_kv);
  const int64_t ldq = (int64_t)a.n_heads * kD, ldk = (int64_t)a.n_kv * kD;
  const int nkb = min(qb, (len - 1) / kBlock) + 1;  // causal: key blocks up to this one
  const uint16_t *kg = a.k + (int64_t)start * ldk + hk * kD;
  const uint16_t *vg = a.v + (int64_t)start * ldk + hk * kD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int wg = warp >> 2, w4 = warp & 3, wtid = threadIdx.x & (kWarps * 32 - 1);
  uint16_t *wbuf = smem + (1 + 4 * wg) * kTileHalves;
  load_tile_async(smem, a.q + (int64_t)(start + q0) * ldq + h * kD, ldq, min(kBlock, len - q0),
                  threadIdx.x, kCtaThreads);
  if (wg < nkb) {
    const int k0 = wg * kBlock;
    load_tile_async(wbuf, kg + (int64_t)k0 * ldk, ldk, min(kBlock, len - k0), wtid, kWarps * 32);
    load_tile_async(wbuf + kTileHalves, vg + (int64_t)k0 * ldk, ldk, min(kBlock, len - k0), wtid,
                    kWarps * 32);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  uint32_t qa[8][4];
  load_a_frags(qa, smem, 16 * w4);

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F, l0 = 0.f, l1 = 0.f;
  const int row0 = q0 + 16 * w4 + g, row1 = row0 + 8;  // query positions in the sequence
  int it = 0;
  for (int kb = wg; kb < nkb; kb += 2, ++it) {
    const int k0 = kb * kBlock;
    if (kb + 2 < nkb) {  // this group's next block into its other buffer
      const int k1 = k0 + 2 * kBlock;
      uint16_t *nb = wbuf + 2 * ((it + 1) & 1) * kTileHalves;
      load_tile_async(nb, kg + (int64_t)k1 * ldk, ldk, min(kBlock, len - k1), wtid, kWarps * 32);
      load_tile_async(nb + kTileHalves, vg + (int64_t)k1 * ldk, ldk, min(kBlock, len - k1), wtid,
                      kWarps * 32);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    wg_sync(wg);  // this block's tiles are in shared memory for the group's warps
    const uint16_t *Ks = wbuf + 2 * (it & 1) * kTileHalves;
    const uint16_t *Vs = Ks + kTileHalves;

    // S = Q K^T for this warp's 16 rows x 64 keys
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kc = 0; kc < 8; ++kc) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bb[4];
        const int kr = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int kcol = kc * 16 + ((lane >> 3) & 1) * 8;
        ldsm4(bb, Ks + kr * kLd + kcol);
        mma16816(s[2 * np], qa[kc], bb[0], bb[1]);
        mma16816(s[2 * np + 1], qa[kc], bb[2], bb[3]);
      }
    }
    // scaled to base 2, masked (keys after the query or past the sequence), online softmax
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + nt * 8 + 2 * t + (e & 1);
        const int row = e < 2 ? row0 : row1;
        float x = s[nt][e] * a.scale_log2;
        if (key > row || key >= len) x = -CUDART_INF_F;
        s[nt][e] = x;
        if (e < 2)
          mx0 = fmaxf(mx0, x);
        else
          mx1 = fmaxf(mx1, x);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float c0 = attn_ex2(m0 - mx0), c1 = attn_ex2(m1 - mx1);  // 0 while m is -inf
    m0 = mx0;
    m1 = mx1;
    l0 *= c0;
    l1 *= c1;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= c0;
      o[i][1] *= c0;
      o[i][2] *= c1;
      o[i][3] *= c1;
    }
    // P (fp16) as the A operand of P V: key chunk kc2 = score tiles 2 kc2, 2 kc2 + 1
    uint32_t pa[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = attn_ex2(s[nt][0] - m0), p1 = attn_ex2(s[nt][1] - m0);
      const float p2 = attn_ex2(s[nt][2] - m1), p3 = attn_ex2(s[nt][3] - m1);
      l0 += p0 + p1;
      l1 += p2 + p3;
      pa[nt >> 1][(nt & 1) * 2] = pack_half2(p0, p1);
      pa[nt >> 1][(nt & 1) * 2 + 1] = pack_half2(p2, p3);
    }
    // O += P V
#pragma unroll
    for (int kc2 = 0; kc2 < 4; ++kc2) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t bb[4];
        const int vr = kc2 * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int vc = dp * 16 + (lane >> 4) * 8;
        ldsm4_t(bb, Vs + vr * kLd + vc);
        mma16816(o[2 * dp], pa[kc2], bb[0], bb[1]);
        mma16816(o[2 * dp + 1], pa[kc2], bb[2], bb[3]);
      }
    }
    wg_sync(wg);  // the group's warps are done with this buffer before it is refilled
  }
  // group 1's state (m, l and O of the same rows) through its now free buffers into group 0
  __syncthreads();
  float *mg = reinterpret_cast<float *>(smem + 5 * kTileHalves);
  const int slot = w4 * 32 + lane;
  if (wg == 1) {
    mg[slot] = m0;
    mg[128 + slot] = m1;
    mg[256 + slot] = l0;
    mg[384 + slot] = l1;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) mg[512 + (nt * 4 + e) * 128 + slot] = o[nt][e];
  }
  __syncthreads();
  if (wg == 1) return;
  {
    const float pm0 = mg[slot], pm1 = mg[128 + slot];
    const float n0 = fmaxf(m0, pm0), n1 = fmaxf(m1, pm1);
    const float a0 = attn_ex2(m0 - n0), b0 = attn_ex2(pm0 - n0);  // 0 for a -inf state
    const float a1 = attn_ex2(m1 - n1), b1 = attn_ex2(pm1 - n1);
    l0 = l0 * a0 + mg[256 + slot] * b0;
    l1 = l1 * a1 + mg[384 + slot] * b1;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      o[nt][0] = o[nt][0] * a0 + mg[512 + (nt * 4 + 0) * 128 + slot] * b0;
      o[nt][1] = o[nt][1] * a0 + mg[512 + (nt * 4 + 1) * 128 + slot] * b0;
      o[nt][2] = o[nt][2] * a1 + mg[512 + (nt * 4 + 2) * 128 + slot] * b1;
      o[nt][3] = o[nt][3] * a1 + mg[512 + (nt * 4 + 3) * 128 + slot] * b1;
    }
    m0 = n0;
    m1 = n1;
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  if (row0 < len) {
    uint32_t *op = reinterpret_cast<uint32_t *>(a.out + (int64_t)(start + row0) * ldq + h * kD);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) op[nt * 4 + t] = pack_half2(o[nt][0] * inv0, o[nt][1] * inv0);
    if (t == 0) a.lse[(int64_t)h * a.total + start + row0] = m0 + __log2f(l0);
  }
  if (row1 < len) {
    uint32_t *op = reinterpret_cast<uint32_t *>(a.out + (int64_t)(start + row1) * ldq + h * kD);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) op[nt * 4 + t] = pack_half2(o[nt][2] * inv1, o[nt][3] * inv1);
    if (t == 0) a.lse[(int64_t)h * a.total + start + row1] = m1 + __log2f(l1);
  }
}

// ---- backward -------------------------------------------------------------------------------
// Three kernels, every sum in a fixed order (deterministic):
//   dq     per (64-query block, head, sequence): D = rowsum(dO o O) for its queries (stored for
//          the next kernel), then over the key blocks up to its own: S = Q K^T, P from the
//          forward's log-sum-exp, dP = dO V^T, dS = P o (dP - D), dQ += dS K; dQ * scale.
//   dkv    per (64-key block, query head, sequence): over the query blocks from its own on:
//          S^T = K Q^T, P^T, dV_h += P^T dO, dP^T = V dO^T, dS^T = P^T o (dP^T - D),
//          dK_h += dS^T Q; fp32 partials dK_h * scale, dV_h per query head.
//   gsum   dK, dV of a key/value head = the sum of its query heads' partials, in head order,
//          rounded once to fp16 (the grouped heads of the reference's repeat_kv).
// dS and P are rounded to fp16 as the operands of their products (as the forward's P).

struct BwdArgs {
  const uint16_t *q, *k, *v, *out, *dout;
  const float *lse;  // [n_heads, total] from the forward
  const int32_t *cu;
  float *delta;      // [n_heads, total] rowsum(dO o O)
  uint16_t *dq;      // [total, n_heads, 128]
  float *dk_part, *dv_part;  // [total, n_heads, 128] per query head
  int64_t total;
  int n_heads, n_kv;
  float scale, scale_log2;
  // With dqkv set (tb_attn_varlen_bwd_rope), the gradients leave through the rotary embedding's
  // backward instead: dqkv[token] = [rot^-1(dq) | rot^-1(dk) | dv] (row stride ld_qkv), each
  // gradient rounded to fp16 first, then rotated back with the token's position
  // (t = pos_idx % seq; a position outside [0, slots) gives a zero row), as tb_rope_tokens_bwd
  // does with the stored fp16 gradients.
  uint16_t *dqkv;
  int64_t ld_qkv;
  const float *cosv, *sinv;  // [seq, 128]
  const int64_t *pos_idx;    // [total]
  int64_t seq, slots;
  FastDiv per_token, seq_div;  // (n_heads + n_kv) * 16 vectors a token; seq (the rotation pass)
};

__global__ void __launch_bounds__(kCtaThreads) attn_bwd_dq_kernel(const __grid_constant__ BwdArgs a) {
  pdl_wait();
  pdl_release();
  extern __shared__ __align__(16) uint16_t smem[];
  __shared__ float d_sh[kBlock];
  // tiles 0, 1: Q, dO; warp group w: tiles 2 + 4w .. 5 + 4w, (K, V) twice. Group w takes key
  // blocks w, w + 2, ...; the two dQ partials are added at the end (group 0's first).
  uint16_t *Qs = smem, *dOs = smem + kTileHalves;
  // grid (heads, batch, query blocks), the last query block first: the longest causal blocks
  // start in the first wave and the shortest fill the tail
  const int qb = (int)(gridDim.z - 1 - blockIdx.z), h = blockIdx.x, b = blockIdx.y;
  const int start = __ldg(a.cu + b), len = __ldg(a.cu + b + 1) - start;
  const int q0 = qb * kBlock;
  if (q0 >= len) return;
  const int hk = h / (a.n_heads / a.n_kv);
  const int64_t ldq = (int64_t)a.n_heads * kD, ldk = (int64_t)a.n_kv * kD;
  const int nq = min(kBlock, len - q0);
  const int nkb = min(qb, (len - 1) / kBlock) + 1;
  const uint16_t *kg = a.k + (int64_t)start * ldk + hk * kD;
  const uint16_t *vg = a.v + (int64_t)start * ldk + hk * kD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int wg = warp >> 2, w4 = warp & 3, wtid = threadIdx.x & (kWarps * 32 - 1);
  uint16_t *wbuf = smem + (2 + 4 * wg) * kTileHalves;
  load_tile_async(Qs, a.q + (int64_t)(start + q0) * ldq + h * kD, ldq, nq, threadIdx.x,
                  kCtaThreads);
  load_tile_async(dOs, a.dout + (int64_t)(start + q0) * ldq + h * kD, ldq, nq, threadIdx.x,
                  kCtaThreads);
  if (wg < nkb) {
    const int k0 = wg * kBlock;
    load_tile_async(wbuf, kg + (int64_t)k0 * ldk, ldk, min(kBlock, len - k0), wtid, kWarps * 32);
    load_tile_async(wbuf + kTileHalves, vg + (int64_t)k0 * ldk, ldk, min(kBlock, len - k0), wtid,
                    kWarps * 32);
  }
  cp_async_commit();
  // D = rowsum(dO o O) of this block's queries: four threads per row, 32 dims each
  {
    const int r = threadIdx.x >> 2, part = threadIdx.x & 3;
    float d = 0.f;
    if (r < nq) {
      const int64_t off = (int64_t)(start + q0 + r) * ldq + h * kD + part * 32;
#pragma unroll
      for (int c = 0; c < 32; c += 8) {
        float x[8], y[8];
        load8h(a.dout + off + c, x);
        load8h(a.out + off + c, y);
#pragma unroll
        for (int e = 0; e < 8; ++e) d = fmaf(x[e], y[e], d);
      }
    }
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    d += __shfl_xor_sync(0xffffffffu, d, 2);
    if (part == 0) {
      d_sh[r] = d;
      if (r < nq) a.delta[(int64_t)h * a.total + start + q0 + r] = d;
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  const int row0 = q0 + 16 * w4 + g, row1 = row0 + 8;
  const float lse0 = row0 < len ? __ldg(a.lse + (int64_t)h * a.total + start + row0) : 0.f;
  const float lse1 = row1 < len ? __ldg(a.lse + (int64_t)h * a.total + start + row1) : 0.f;
  const float d0 = d_sh[16 * w4 + g], d1 = d_sh[16 * w4 + g + 8];
  float dq[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  const int ar = 16 * w4 + (lane & 7) + ((lane >> 3) & 1) * 8, ac = (lane >> 4) * 8;
  int it = 0;
  for (int kb = wg; kb < nkb; kb += 2, ++it) {
    const int k0 = kb * kBlock;
    if (kb + 2 < nkb) {
      const int k1 = k0 + 2 * kBlock;
      uint16_t *nb = wbuf + 2 * ((it + 1) & 1) * kTileHalves;
      load_tile_async(nb, kg + (int64_t)k1 * ldk, ldk, min(kBlock, len - k1), wtid, kWarps * 32);
      load_tile_async(nb + kTileHalves, vg + (int64_t)k1 * ldk, ldk, min(kBlock, len - k1), wtid,
                      kWarps * 32);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    wg_sync(wg);
    const uint16_t *Ks = wbuf + 2 * (it & 1) * kTileHalves;
    const uint16_t *Vs = Ks + kTileHalves;
    float s[8][4], dp[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
      dp[i][0] = dp[i][1] = dp[i][2] = dp[i][3] = 0.f;
    }
#pragma unroll
    for (int kc = 0; kc < 8; ++kc) {
      uint32_t qa[4], da[4];
      ldsm4(qa, Qs + ar * kLd + kc * 16 + ac);
      ldsm4(da, dOs + ar * kLd + kc * 16 + ac);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bk[4], bv[4];
        const int kr = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int kcol = kc * 16 + ((lane >> 3) & 1) * 8;
        ldsm4(bk, Ks + kr * kLd + kcol);
        ldsm4(bv, Vs + kr * kLd + kcol);
        mma16816(s[2 * np], qa, bk[0], bk[1]);
        mma16816(s[2 * np + 1], qa, bk[2], bk[3]);
        mma16816(dp[2 * np], da, bv[0], bv[1]);
        mma16816(dp[2 * np + 1], da, bv[2], bv[3]);
      }
    }
    // dS = P o (dP - D) as fp16 A fragments over the 64 keys
    uint32_t dsa[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float ds[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + nt * 8 + 2 * t + (e & 1);
        const int row = e < 2 ? row0 : row1;
        const float p = (key > row || key >= len || row >= len)
                            ? 0.f
                            : attn_ex2(s[nt][e] * a.scale_log2 - (e < 2 ? lse0 : lse1));
        ds[e] = p * (dp[nt][e] - (e < 2 ? d0 : d1));
      }
      dsa[nt >> 1][(nt & 1) * 2] = pack_half2(ds[0], ds[1]);
      dsa[nt >> 1][(nt & 1) * 2 + 1] = pack_half2(ds[2], ds[3]);
    }
    // dQ += dS K  (K as the [key, dim] B operand: transposed fragments)
#pragma unroll
    for (int kc2 = 0; kc2 < 4; ++kc2) {
#pragma unroll
      for (int dpi = 0; dpi < 8; ++dpi) {
        uint32_t bb[4];
        const int kr = kc2 * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int kcl = dpi * 16 + (lane >> 4) * 8;
        ldsm4_t(bb, Ks + kr * kLd + kcl);
        mma16816(dq[2 * dpi], dsa[kc2], bb[0], bb[1]);
        mma16816(dq[2 * dpi + 1], dsa[kc2], bb[2], bb[3]);
      }
    }
    wg_sync(wg);
  }
  // group 1's dQ partial through its now free buffers, added to group 0's
  __syncthreads();
  float *mg = reinterpret_cast<float *>(smem + 6 * kTileHalves);
  const int slot = w4 * 32 + lane;
  if (wg == 1) {
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) mg[(nt * 4 + e) * 128 + slot] = dq[nt][e];
  }
  __syncthreads();
  if (wg == 1) return;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) dq[nt][e] += mg[(nt * 4 + e) * 128 + slot];
  // with dqkv set (the backward through the rotary embedding), the scaled fp16 dQ goes to
  // dqkv's q columns unrotated; attn_bwd_gsum_rope_kernel rotates it in place
  uint16_t *dq_out = a.dqkv != nullptr ? a.dqkv : a.dq;
  const int64_t ld_out = a.dqkv != nullptr ? a.ld_qkv : ldq;
  if (row0 < len) {
    uint32_t *op = reinterpret_cast<uint32_t *>(dq_out + (int64_t)(start + row0) * ld_out + h * kD);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
      op[nt * 4 + t] = pack_half2(dq[nt][0] * a.scale, dq[nt][1] * a.scale);
  }
  if (row1 < len) {
    uint32_t *op = reinterpret_cast<uint32_t *>(dq_out + (int64_t)(start + row1) * ld_out + h * kD);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
      op[nt * 4 + t] = pack_half2(dq[nt][2] * a.scale, dq[nt][3] * a.scale);
  }
}

__global__ void __launch_bounds__(kCtaThreads) attn_bwd_dkv_kernel(const __grid_constant__ BwdArgs a) {
  pdl_wait();
  pdl_release();
  extern __shared__ __align__(16) uint16_t smem[];
  __shared__ float lse_sh[2][2][kBlock], d_sh[2][2][kBlock];  // [group][buffer][query]
  // tiles 0, 1: K, V; warp group w: tiles 2 + 4w .. 5 + 4w, (Q, dO) twice. Group w takes query
  // blocks kb + w, kb + w + 2, ...; the two dK / dV partials are added at the end (group 0's
  // first).
  uint16_t *Ks = smem, *Vs = smem + kTileHalves;
  // grid (heads, batch, key blocks), key block 0 (which every query block sees) first
  const int kb = blockIdx.z, h = blockIdx.x, b = blockIdx.y;
  const int start = __ldg(a.cu + b), len = __ldg(a.cu + b + 1) - start;
  const int k0 = kb * kBlock;
  if (k0 >= len) return;
  const int hk = h / (a.n_heads / a.n_kv);
  const int64_t ldq = (int64_t)a.n_heads * kD, ldk = (int64_t)a.n_kv * kD;
  const int nqb = (len - 1) / kBlock + 1;  // query blocks kb .. nqb - 1 see these keys
  const uint16_t *qg = a.q + (int64_t)start * ldq + h * kD;
  const uint16_t *dog = a.dout + (int64_t)start * ldq + h * kD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int wg = warp >> 2, w4 = warp & 3, wtid = threadIdx.x & (kWarps * 32 - 1);
  uint16_t *wbuf = smem + (2 + 4 * wg) * kTileHalves;
  load_tile_async(Ks, a.k + (int64_t)(start + k0) * ldk + hk * kD, ldk, min(kBlock, len - k0),
                  threadIdx.x, kCtaThreads);
  load_tile_async(Vs, a.v + (int64_t)(start + k0) * ldk + hk * kD, ldk, min(kBlock, len - k0),
                  threadIdx.x, kCtaThreads);
  if (kb + wg < nqb) {
    const int q0 = (kb + wg) * kBlock;
    load_tile_async(wbuf, qg + (int64_t)q0 * ldq, ldq, min(kBlock, len - q0), wtid, kWarps * 32);
    load_tile_async(wbuf + kTileHalves, dog + (int64_t)q0 * ldq, ldq, min(kBlock, len - q0), wtid,
                    kWarps * 32);
    if (wtid < kBlock) {
      const int qi = q0 + wtid;
      lse_sh[wg][0][wtid] = qi < len ? __ldg(a.lse + (int64_t)h * a.total + start + qi) : 0.f;
      d_sh[wg][0][wtid] = qi < len ? __ldg(a.delta + (int64_t)h * a.total + start + qi) : 0.f;
    }
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  const int key0 = k0 + 16 * w4 + g, key1 = key0 + 8;
  float dk[16][4], dv[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
    dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  }
  const int ar = 16 * w4 + (lane & 7) + ((lane >> 3) & 1) * 8, ac = (lane >> 4) * 8;
  int it = 0;
  for (int qb = kb + wg; qb < nqb; qb += 2, ++it) {
    const int q0 = qb * kBlock;
    if (qb + 2 < nqb) {  // this group's next query block into its other buffer
      const int q1 = q0 + 2 * kBlock;
      uint16_t *nb = wbuf + 2 * ((it + 1) & 1) * kTileHalves;
      load_tile_async(nb, qg + (int64_t)q1 * ldq, ldq, min(kBlock, len - q1), wtid, kWarps * 32);
      load_tile_async(nb + kTileHalves, dog + (int64_t)q1 * ldq, ldq, min(kBlock, len - q1), wtid,
                      kWarps * 32);
      cp_async_commit();
      if (wtid < kBlock) {
        const int qi = q1 + wtid;
        lse_sh[wg][(it + 1) & 1][wtid] =
            qi < len ? __ldg(a.lse + (int64_t)h * a.total + start + qi) : 0.f;
        d_sh[wg][(it + 1) & 1][wtid] =
            qi < len ? __ldg(a.delta + (int64_t)h * a.total + start + qi) : 0.f;
      }
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    wg_sync(wg);
    const uint16_t *Qs = wbuf + 2 * (it & 1) * kTileHalves;
    const uint16_t *dOs = Qs + kTileHalves;
    const float *lse = lse_sh[wg][it & 1], *dd = d_sh[wg][it & 1];
    // S^T = K Q^T and dP^T = V dO^T: 16 keys x 64 queries per warp
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.f;
      dpt[i][0] = dpt[i][1] = dpt[i][2] = dpt[i][3] = 0.f;
    }
#pragma unroll
    for (int kc = 0; kc < 8; ++kc) {
      uint32_t ka[4], va[4];
      ldsm4(ka, Ks + ar * kLd + kc * 16 + ac);
      ldsm4(va, Vs + ar * kLd + kc * 16 + ac);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bq[4], bd[4];
        const int qr = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int qcol = kc * 16 + ((lane >> 3) & 1) * 8;
        ldsm4(bq, Qs + qr * kLd + qcol);
        ldsm4(bd, dOs + qr * kLd + qcol);
        mma16816(st[2 * np], ka, bq[0], bq[1]);
        mma16816(st[2 * np + 1], ka, bq[2], bq[3]);
        mma16816(dpt[2 * np], va, bd[0], bd[1]);
        mma16816(dpt[2 * np + 1], va, bd[2], bd[3]);
      }
    }
    // P^T and dS^T as fp16 A fragments over the 64 queries
    uint32_t pa[4][4], dsa[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float p[4], ds[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qcol = nt * 8 + 2 * t + (e & 1);
        const int qi = q0 + qcol;
        const int key = e < 2 ? key0 : key1;
        p[e] = (qi < key || qi >= len) ? 0.f : attn_ex2(st[nt][e] * a.scale_log2 - lse[qcol]);
        ds[e] = p[e] * (dpt[nt][e] - dd[qcol]);
      }
      pa[nt >> 1][(nt & 1) * 2] = pack_half2(p[0], p[1]);
      pa[nt >> 1][(nt & 1) * 2 + 1] = pack_half2(p[2], p[3]);
      dsa[nt >> 1][(nt & 1) * 2] = pack_half2(ds[0], ds[1]);
      dsa[nt >> 1][(nt & 1) * 2 + 1] = pack_half2(ds[2], ds[3]);
    }
    // dV += P^T dO, dK += dS^T Q  (dO, Q as [query, dim] B operands: transposed fragments)
#pragma unroll
    for (int kc2 = 0; kc2 < 4; ++kc2) {
#pragma unroll
      for (int dpi = 0; dpi < 8; ++dpi) {
        uint32_t bd[4], bq[4];
        const int r = kc2 * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dpi * 16 + (lane >> 4) * 8;
        ldsm4_t(bd, dOs + r * kLd + c);
        ldsm4_t(bq, Qs + r * kLd + c);
        mma16816(dv[2 * dpi], pa[kc2], bd[0], bd[1]);
        mma16816(dv[2 * dpi + 1], pa[kc2], bd[2], bd[3]);
        mma16816(dk[2 * dpi], dsa[kc2], bq[0], bq[1]);
        mma16816(dk[2 * dpi + 1], dsa[kc2], bq[2], bq[3]);
      }
    }
    wg_sync(wg);
  }
  // group 1's dK / dV partials through its now free buffers, added to group 0's
  __syncthreads();
  float *mg = reinterpret_cast<float *>(smem + 6 * kTileHalves);
  const int slot = w4 * 32 + lane;
  if (wg == 1) {
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        mg[(nt * 4 + e) * 128 + slot] = dk[nt][e];
        mg[8192 + (nt * 4 + e) * 128 + slot] = dv[nt][e];
      }
  }
  __syncthreads();
  if (wg == 1) return;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      dk[nt][e] += mg[(nt * 4 + e) * 128 + slot];
      dv[nt][e] += mg[8192 + (nt * 4 + e) * 128 + slot];
    }
  // fp32 partials of this query head: rows key0 / key1, 8 columns per n-tile pair
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const int key = hf == 0 ? key0 : key1;
    if (key >= len) continue;
    float *pk = a.dk_part + (int64_t)(start + key) * ldq + h * kD;
    float *pv = a.dv_part + (int64_t)(start + key) * ldq + h * kD;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      *reinterpret_cast<float2 *>(pk + nt * 8 + 2 * t) =
          make_float2(dk[nt][2 * hf] * a.scale, dk[nt][2 * hf + 1] * a.scale);
      *reinterpret_cast<float2 *>(pv + nt * 8 + 2 * t) = make_float2(dv[nt][2 * hf], dv[nt][2 * hf + 1]);
    }
  }
}

// dK, dV fp16 [total, n_kv, 128] = sums of the fp32 partials of each group's query heads, in
// head order. A thread takes 4 columns of one (token, key/value head) and issues every group
// member's loads before adding (groups of up to kMaxGroup heads; larger groups loop).
constexpr int kMaxGroup = 8;

__global__ void __launch_bounds__(256) attn_bwd_gsum_kernel(const float *__restrict__ dk_part,
                                                            const float *__restrict__ dv_part,
                                                            uint16_t *__restrict__ dk,
                                                            uint16_t *__restrict__ dv,
                                                            int64_t total, int n_heads, int n_kv) {
  pdl_wait();
  pdl_release();
  const int group = n_heads / n_kv;
  const int64_t nvec = total * n_kv * (kD / 4);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tok = i / (n_kv * (kD / 4));
    const int rem = (int)(i - tok * (n_kv * (kD / 4)));
    const int hk = rem / (kD / 4), c = (rem % (kD / 4)) * 4;
    const int64_t src = tok * (int64_t)n_heads * kD + (int64_t)hk * group * kD + c;
    float4 sk = make_float4(0.f, 0.f, 0.f, 0.f), sv = sk;
    for (int j0 = 0; j0 < group; j0 += kMaxGroup) {
      float4 xk[kMaxGroup], xv[kMaxGroup];
#pragma unroll
      for (int j = 0; j < kMaxGroup; ++j) {
        if (j0 + j < group) {
          xk[j] = __ldg(reinterpret_cast<const float4 *>(dk_part + src + (int64_t)(j0 + j) * kD));
          xv[j] = __ldg(reinterpret_cast<const float4 *>(dv_part + src + (int64_t)(j0 + j) * kD));
        }
      }
#pragma unroll
      for (int j = 0; j < kMaxGroup; ++j) {
        if (j0 + j < group) {
          sk.x += xk[j].x; sk.y += xk[j].y; sk.z += xk[j].z; sk.w += xk[j].w;
          sv.x += xv[j].x; sv.y += xv[j].y; sv.z += xv[j].z; sv.w += xv[j].w;
        }
      }
    }
    const int64_t dst = tok * (int64_t)n_kv * kD + (int64_t)hk * kD + c;
    *reinterpret_cast<uint2 *>(dk + dst) = make_uint2(pack_half2(sk.x, sk.y), pack_half2(sk.z, sk.w));
    *reinterpret_cast<uint2 *>(dv + dst) = make_uint2(pack_half2(sv.x, sv.y), pack_half2(sv.z, sv.w));
  }
}

// The backward through the rotary embedding, finished in one pass over dqkv: a thread takes 4
// columns c..c+3 and c+64..c+67 of one head slot of one token. Slots 0 .. n_heads-1 are the q
// heads: the dQ kernel left fp16 dQ in dqkv's q columns, rotated back here in place. Slots
// n_heads .. n_heads+n_kv-1 are the key/value heads: the grouped query heads' fp32 dK and dV
// partials summed in head order, dK rotated back, dV copied. The rotation is
// tb_rope_tokens_bwd's: each gradient rounded to fp16, then (g1 c1 + g2 s2, g2 c2 - g1 s1) with
// the table row t = pos_idx[token] % seq; a token without a position gets zeros.
__global__ void __launch_bounds__(256) attn_bwd_gsum_rope_kernel(const __grid_constant__ BwdArgs a) {
  pdl_wait();
  pdl_release();
  const int group = a.n_heads / a.n_kv;
  // 16 vectors of 4 in the first half of a head; 32-bit items (the host keeps their count below 2^31), divisions by invariant divisors
  const uint32_t nvec = (uint32_t)a.total * a.per_token.d;
  const int64_t slots = a.slots;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += gridDim.x * blockDim.x) {
    uint32_t tok32, rem;
    a.per_token.divmod(i, tok32, rem);
    const int64_t tok = tok32;
    const int slot = (int)(rem >> 4), c = (int)(rem & 15) * 4;
    const int64_t pos = __ldg(a.pos_idx + tok);
    uint32_t tq, tr;
    a.seq_div.divmod((uint32_t)pos, tq, tr);
    const int tp = (pos >= 0 && pos < slots) ? (int)tr : -1;
    uint16_t *row = a.dqkv + tok * a.ld_qkv;
    float g1[4], g2[4];
    float v1[4] = {0.f, 0.f, 0.f, 0.f}, v2[4] = {0.f, 0.f, 0.f, 0.f};
    uint16_t *dst;
    const bool is_q = slot < a.n_heads;
    if (is_q) {
      dst = row + (int64_t)slot * kD + c;
      const uint2 x1 = *reinterpret_cast<const uint2 *>(dst);
      const uint2 x2 = *reinterpret_cast<const uint2 *>(dst + 64);
      const float2 p0 = unpack_half2(x1.x), p1 = unpack_half2(x1.y);
      const float2 p2 = unpack_half2(x2.x), p3 = unpack_half2(x2.y);
      g1[0] = p0.x; g1[1] = p0.y; g1[2] = p1.x; g1[3] = p1.y;
      g2[0] = p2.x; g2[1] = p2.y; g2[2] = p3.x; g2[3] = p3.y;
    } else {
      const int hk = slot - a.n_heads;
      const int64_t src = tok * (int64_t)a.n_heads * kD + (int64_t)hk * group * kD + c;
      float k1[4] = {0.f, 0.f, 0.f, 0.f}, k2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
      for (int j = 0; j < group; ++j) {
        const int64_t o = src + (int64_t)j * kD;
        const float4 xk1 = __ldg(reinterpret_cast<const float4 *>(a.dk_part + o));
        const float4 xk2 = __ldg(reinterpret_cast<const float4 *>(a.dk_part + o + 64));
        const float4 xv1 = __ldg(reinterpret_cast<const float4 *>(a.dv_part + o));
        const float4 xv2 = __ldg(reinterpret_cast<const float4 *>(a.dv_part + o + 64));
        k1[0] += xk1.x; k1[1] += xk1.y; k1[2] += xk1.z; k1[3] += xk1.w;
        k2[0] += xk2.x; k2[1] += xk2.y; k2[2] += xk2.z; k2[3] += xk2.w;
        v1[0] += xv1.x; v1[1] += xv1.y; v1[2] += xv1.z; v1[3] += xv1.w;
        v2[0] += xv2.x; v2[1] += xv2.y; v2[2] += xv2.z; v2[3] += xv2.w;
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {  // the fp16 gradients the separate rotation would read
        g1[e] = __half2float(__float2half_rn(k1[e]));
        g2[e] = __half2float(__float2half_rn(k2[e]));
      }
      dst = row + (int64_t)(a.n_heads + hk) * kD + c;
      uint16_t *dv = row + (int64_t)(a.n_heads + a.n_kv + hk) * kD + c;
      if (tp < 0) {
#pragma unroll
        for (int e = 0; e < 4; ++e) v1[e] = v2[e] = 0.f;
      }
      *reinterpret_cast<uint2 *>(dv) =
          make_uint2(pack_half2(v1[0], v1[1]), pack_half2(v1[2], v1[3]));
      *reinterpret_cast<uint2 *>(dv + 64) =
          make_uint2(pack_half2(v2[0], v2[1]), pack_half2(v2[2], v2[3]));
    }
    float o1[4] = {0.f, 0.f, 0.f, 0.f}, o2[4] = {0.f, 0.f, 0.f, 0.f};
    if (tp >= 0) {
      const float *cr = a.cosv + (int64_t)tp * kD + c, *sr = a.sinv + (int64_t)tp * kD + c;
      const float4 c1 = __ldg(reinterpret_cast<const float4 *>(cr));
      const float4 c2 = __ldg(reinterpret_cast<const float4 *>(cr + 64));
      const float4 s1 = __ldg(reinterpret_cast<const float4 *>(sr));
      const float4 s2 = __ldg(reinterpret_cast<const float4 *>(sr + 64));
      const float cc1[4] = {c1.x, c1.y, c1.z, c1.w}, cc2[4] = {c2.x, c2.y, c2.z, c2.w};
      const float ss1[4] = {s1.x, s1.y, s1.z, s1.w}, ss2[4] = {s2.x, s2.y, s2.z, s2.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        o1[e] = g1[e] * cc1[e] + g2[e] * ss2[e];
        o2[e] = g2[e] * cc2[e] - g1[e] * ss1[e];
      }
    }
    *reinterpret_cast<uint2 *>(dst) = make_uint2(pack_half2(o1[0], o1[1]), pack_half2(o1[2], o1[3]));
    *reinterpret_cast<uint2 *>(dst + 64) =
        make_uint2(pack_half2(o2[0], o2[1]), pack_half2(o2[2], o2[3]));
  }
}

int check_attn(const char *what, const void *q, const void *k, const void *v, const int32_t *cu,
               int64_t batch, int64_t total, int64_t max_len, int32_t n_heads, int32_t n_kv,
               int32_t head_dim) {
  if (head_dim != kD)
    return set_error(TB_EINVAL, "%s: head_dim %d (the kernels take %d)", what, head_dim, kD);
  if (batch < 0 || total < 0 || max_len < 0 || n_heads < 1 || n_kv < 1 || n_heads % n_kv)
    return set_error(TB_EINVAL, "%s: batch %lld total %lld max_len %lld heads %d/%d", what,
                     (long long)batch, (long long)total, (long long)max_len, n_heads, n_kv);
  if (batch > 65535 || n_heads > 65535 || (max_len + kBlock - 1) / kBlock > 65535 ||
      total > (1LL << 31))
    return set_error(TB_EINVAL, "%s: sizes too large", what);
  if (!q || !k || !v || !cu) return set_error(TB_EINVAL, "%s: q, k, v, cu_seqlens required", what);
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16))
    return set_error(TB_EALIGN, "%s: q, k, v must be 16-byte aligned", what);
  return TB_OK;
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" int tb_attn_varlen_fwd(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                                  const int32_t *cu_seqlens, uint16_t *out, float *lse,
                                  int64_t batch, int64_t total, int64_t max_len, int32_t n_heads,
                                  int32_t n_kv, int32_t head_dim, float scale, void *stream) {
  int rc = check_attn("attn_varlen_fwd", q, k, v, cu_seqlens, batch, total, max_len, n_heads,
                      n_kv, head_dim);
  if (rc != TB_OK) return rc;
  if (!out || !lse) return set_error(TB_EINVAL, "attn_varlen_fwd: out and lse required");
  if (!aligned(out, 16)) return set_error(TB_EALIGN, "attn_varlen_fwd: out must be 16-byte aligned");
  if (batch == 0 || total == 0 || max_len == 0) return TB_OK;
  const size_t smem = 9 * kTileHalves * sizeof(uint16_t);
  // set on every call: the attribute belongs to the current device
  if (cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return check_launch("attn_varlen_fwd attribute");
  FwdArgs a{q, k, v, cu_seqlens, out, lse, total, n_heads, n_kv, scale * 1.4426950408889634f};
  const dim3 grid((unsigned)n_heads, (unsigned)batch, (unsigned)((max_len + kBlock - 1) / kBlock));
  return launch("attn_varlen_fwd", attn_fwd_kernel, grid, kCtaThreads, smem, as_stream(stream), a);
}

extern "C" int tb_attn_varlen_bwd(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                                  const uint16_t *out, const uint16_t *dout, const float *lse,
                                  const int32_t *cu_seqlens, uint16_t *dq, uint16_t *dk,
                                  uint16_t *dv, float *delta, float *dk_part, float *dv_part,
                                  int64_t batch, int64_t total, int64_t max_len, int32_t n_heads,
                                  int32_t n_kv, int32_t head_dim, float scale, void *stream) {
  int rc = check_attn("attn_varlen_bwd", q, k, v, cu_seqlens, batch, total, max_len, n_heads,
                      n_kv, head_dim);
  if (rc != TB_OK) return rc;
  if (!out || !dout || !lse || !dq || !dk || !dv || !delta || !dk_part || !dv_part)
    return set_error(TB_EINVAL, "attn_varlen_bwd: every buffer is required");
  if (!aligned(out, 16) || !aligned(dout, 16) || !aligned(dq, 16) || !aligned(dk, 16) ||
      !aligned(dv, 16) || !aligned(dk_part, 16) || !aligned(dv_part, 16))
    return set_error(TB_EALIGN, "attn_varlen_bwd: 16-byte aligned buffers are required");
  if (batch == 0 || total == 0 || max_len == 0) return TB_OK;
  const size_t smem = 10 * kTileHalves * sizeof(uint16_t);
  if (cudaFuncSetAttribute(attn_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess ||
      cudaFuncSetAttribute(attn_bwd_dkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return check_launch("attn_varlen_bwd attribute");
  BwdArgs a{q,     k,      v,       out,     dout,    lse,     cu_seqlens,
            delta, dq,     dk_part, dv_part, total,   n_heads, n_kv,
            scale, scale * 1.4426950408889634f, nullptr, 0, nullptr, nullptr, nullptr, 0, 0};
  const dim3 grid((unsigned)n_heads, (unsigned)batch, (unsigned)((max_len + kBlock - 1) / kBlock));
  cudaStream_t st = as_stream(stream);
  rc = launch("attn_varlen_bwd dq", attn_bwd_dq_kernel, grid, kCtaThreads, smem, st, a);
  if (rc != TB_OK) return rc;
  rc = launch("attn_varlen_bwd dkv", attn_bwd_dkv_kernel, grid, kCtaThreads, smem, st, a);
  if (rc != TB_OK) return rc;
  const int64_t nvec = total * n_kv * (kD / 4);
  int64_t blocks = (nvec + 255) / 256;
  if (blocks > (int64_t)sm_count() * 8) blocks = (int64_t)sm_count() * 8;
  return launch("attn_varlen_bwd gsum", attn_bwd_gsum_kernel, (unsigned)blocks, 256, 0, st,
                (const float *)dk_part, (const float *)dv_part, dk, dv, total, (int)n_heads,
                (int)n_kv);
}

// tb_attn_varlen_bwd whose gradients leave through the rotary embedding's backward: writes
// dqkv [total, (n_heads + 2 n_kv) * 128] (row stride ld_qkv) = what tb_rope_tokens_bwd writes
// from the dq, dk, dv tb_attn_varlen_bwd would write, without storing those.
extern "C" int tb_attn_varlen_bwd_rope(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                                       const uint16_t *out, const uint16_t *dout, const float *lse,
                                       const int32_t *cu_seqlens, const float *cos,
                                       const float *sin, const int64_t *pos_idx, int64_t seq,
                                       int64_t slots, uint16_t *dqkv, int64_t ld_qkv,
                                       float *delta, float *dk_part, float *dv_part,
                                       int64_t batch, int64_t total, int64_t max_len,
                                       int32_t n_heads, int32_t n_kv, int32_t head_dim,
                                       float scale, void *stream) {
  int rc = check_attn("attn_varlen_bwd_rope", q, k, v, cu_seqlens, batch, total, max_len,
                      n_heads, n_kv, head_dim);
  if (rc != TB_OK) return rc;
  if (!out || !dout || !lse || !cos || !sin || !pos_idx || !dqkv || !delta || !dk_part ||
      !dv_part)
    return set_error(TB_EINVAL, "attn_varlen_bwd_rope: every buffer is required");
  if (seq <= 0 || slots < 0 || slots > 0x7fffffffLL || seq > 0x7fffffffLL ||
      ld_qkv < (int64_t)(n_heads + 2 * n_kv) * kD || ld_qkv % 8 != 0 ||
      total * (n_heads + n_kv) * (kD / 8) >= (1LL << 31))
    return set_error(TB_EINVAL, "attn_varlen_bwd_rope: seq %lld slots %lld ld_qkv %lld",
                     (long long)seq, (long long)slots, (long long)ld_qkv);
  if (!aligned(out, 16) || !aligned(dout, 16) || !aligned(dqkv, 16) || !aligned(dk_part, 16) ||
      !aligned(dv_part, 16) || !aligned(cos, 16) || !aligned(sin, 16))
    return set_error(TB_EALIGN, "attn_varlen_bwd_rope: 16-byte aligned buffers are required");
  if (batch == 0 || total == 0 || max_len == 0) return TB_OK;
  const size_t smem = 10 * kTileHalves * sizeof(uint16_t);
  if (cudaFuncSetAttribute(attn_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess ||
      cudaFuncSetAttribute(attn_bwd_dkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return check_launch("attn_varlen_bwd_rope attribute");
  BwdArgs a{q,     k,      v,       out,     dout,    lse,     cu_seqlens,
            delta, nullptr, dk_part, dv_part, total,  n_heads, n_kv,
            scale, scale * 1.4426950408889634f, dqkv, ld_qkv, cos, sin, pos_idx, seq, slots};
  const dim3 grid((unsigned)n_heads, (unsigned)batch, (unsigned)((max_len + kBlock - 1) / kBlock));
  cudaStream_t st = as_stream(stream);
  rc = launch("attn_varlen_bwd_rope dq", attn_bwd_dq_kernel, grid, kCtaThreads, smem, st, a);
  if (rc != TB_OK) return rc;
  rc = launch("attn_varlen_bwd_rope dkv", attn_bwd_dkv_kernel, grid, kCtaThreads, smem, st, a);
  if (rc != TB_OK) return rc;
  const int64_t nvec = total * (n_heads + n_kv) * (kD / 8);
  int64_t blocks = (nvec + 255) / 256;
  if (blocks > (int64_t)sm_count() * 8) blocks = (int64_t)sm_count() * 8;
  a.per_token = FastDiv((uint32_t)((n_heads + n_kv) * (kD / 8)));
  a.seq_div = FastDiv((uint32_t)seq);
  return launch("attn_varlen_bwd_rope rotate", attn_bwd_gsum_rope_kernel, (unsigned)blocks, 256,
                0, st, a);
}
