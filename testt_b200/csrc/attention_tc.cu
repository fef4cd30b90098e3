// Variable-length causal attention forward on the 5th-generation tensor cores (tcgen05 with
// TMEM accumulators, TMA tiles). Same contract as tb_attn_varlen_fwd (attention.cu): the
// decoder layer's attention of solution/model.py:242-247 restricted to each sequence's real
// rows, grouped key/value heads, head dim 128, writing O (fp16, token-major) and the base-2
// log-sum-exp of the scaled scores per (head, query).
//
// A CTA takes 128 queries of one head of one sequence; the key tiles (128 keys) up to its own
// (causal). Warps:
//   warp 8     TMA producer: the Q tile once, then K and V tiles through a 4-slot ring in the
//              order the MMA uses them
//   warp 9     TMEM allocation and the MMA issuer:
//                S = Q K^T     M128 N128 K128, both operands K-major in shared memory
//                O += P V      M128 N128 K128, P read from TMEM, V MN-major in shared memory
//   warps 0-7  softmax and epilogue: warps w and w + 4 share TMEM lane quarter w % 4, so a
//              row's two threads each see the whole row (no shuffles); both take the row
//              maximum over all 128 keys of a tile, each forms P for its 64 keys and rescales and
//              writes its 64 columns of O; their row sums are added once, at the end
// One pass over the key tiles with an online softmax in base 2. S is double-buffered in TMEM, so
// the MMA computes the next tile's scores while the softmax warps work on the current one. The
// row maximum m that P = 2^(s - m) is taken against moves only when a tile's maximum exceeds it
// by more than 2^8 (then O, in TMEM, is rescaled by the softmax warps once the last P V has
// finished); otherwise P values up to 256 are used against the older maximum, which changes
// nothing but rounding: the row sum l is formed from the same fp32 values, and the log-sum-exp
// is m + log2(l) for whichever m was used.
// TMEM columns: S0 0-127, S1 128-255, P 256-319 (fp16 pairs), O 384-511.
//
// Every mbarrier wait is bounded (mbar_wait); a role that gives up sets the CTA's error flag and
// leaves its loop, every role meets at the final barrier and TMEM is always released. No
// multicast is used.
#include <cuda.h>
#include <math_constants.h>

#include "common.cuh"

namespace tb {
namespace {

constexpr int kD = 128;                       // head dimension
constexpr int kTile = 128;                    // queries per CTA, keys per tile
constexpr int kRing = 4;                      // K / V tiles in flight
constexpr int kBoxBytes = kTile * 64 * 2;     // 16 KB: 128 rows x 64 columns (one TMA box)
constexpr int kTileBytes = 2 * kBoxBytes;     // 32 KB: 128 rows x 128 columns
constexpr int kThreads = 320;
constexpr int kTmemCols = 512;
constexpr uint32_t kColS = 0, kColP = 256, kColO = 384;  // S buffer b at kColS + 128 b
constexpr float kRescaleAt = 8.f;  // log2 of the largest P the kept maximum may produce

// M = 128, N = 128, fp16 inputs, fp32 accumulation; S: A and B K-major
constexpr uint32_t kIdescS = (1u << 4) | ((uint32_t)(kTile >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
// O += P V: A from TMEM (K-major), B = V MN-major (bit 16)
constexpr uint32_t kIdescO =
    (1u << 4) | (1u << 16) | ((uint32_t)(kD >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

struct Smem {
  alignas(1024) uint8_t q[kTileBytes];
  alignas(1024) uint8_t ring[kRing][kTileBytes];
  uint64_t q_full, ring_full[kRing], ring_empty[kRing];
  uint64_t s_full[2], s_read[2], p_full, p_free, o_full, mma_done;
  float l_pair[2][128];  // the two half-row sums of P (epilogue)
  uint32_t tmem_base;
  volatile int error;
};

static_assert(sizeof(Smem) + 1024 <= 232448, "shared memory of an attention CTA");

struct TcArgs {
  const int32_t *cu;
  uint16_t *out;
  float *lse;  // [n_heads, total]
  int64_t total;
  int n_heads, n_kv;
  float scale_log2;
};

// K-major, 128-byte swizzle: SBO 1024 bytes between 8-row atoms, sm_100 descriptor version
__device__ __forceinline__ uint64_t desc_k(uint32_t addr) {
  uint64_t d = (uint64_t)((addr >> 4) & 0x3fff);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// MN-major, 128-byte swizzle: LBO = one box between the two 64-column halves of N, SBO 1024
// bytes between 8-row groups along K
__device__ __forceinline__ uint64_t desc_mn(uint32_t addr) {
  uint64_t d = (uint64_t)((addr >> 4) & 0x3fff);
  d |= (uint64_t)(kBoxBytes >> 4) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int c0, int c1,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::
                   "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ float ex2a(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Tile i of the producer / MMA order: K0, then for each key tile kt the next tile's K (when
// there is one) before V(kt), so the scores of tile kt + 1 are computed before P(kt) V(kt):
//   K0, K1, V0, K2, V1, ..., K(n-1), V(n-2), V(n-1)
__device__ __forceinline__ void tile_of(int i, int n, bool &is_v, int &kt) {
  if (i == 0) {
    is_v = false;
    kt = 0;
  } else if (i == 2 * n - 1) {
    is_v = true;
    kt = n - 1;
  } else {
    // i = 1, 2 -> K1, V0; i = 3, 4 -> K2, V1; ...
    is_v = (i & 1) == 0;
    kt = is_v ? (i >> 1) - 1 : (i + 1) >> 1;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap map_q,
                       const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v, const __grid_constant__ TcArgs a) {
  pdl_wait();
  pdl_release();
  // grid (heads, sequences, query tiles), the last query tile first (the most key tiles)
  const int qt = (int)(gridDim.z - 1 - blockIdx.z), h = blockIdx.x, b = blockIdx.y;
  const int start = __ldg(a.cu + b), len = __ldg(a.cu + b + 1) - start;
  const int q0 = qt * kTile;
  if (q0 >= len) return;  // the whole CTA, before any barrier or allocation
  extern __shared__ uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                        ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = h / (a.n_heads / a.n_kv);
  const int n = min(qt, (len - 1) / kTile) + 1;  // key tiles 0 .. n-1 (causal)
  const int tiles = 2 * n;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&sm.ring_full[s], 1);
      mbar_init(&sm.ring_empty[s], 1);
    }
    for (int b2 = 0; b2 < 2; ++b2) {
      mbar_init(&sm.s_full[b2], 1);
      mbar_init(&sm.s_read[b2], 8);  // the 8 softmax warps
    }
    mbar_init(&sm.p_full, 8);
    mbar_init(&sm.p_free, 1);
    mbar_init(&sm.o_full, 1);
    mbar_init(&sm.mma_done, 1);
    sm.error = 0;
    mbar_init_fence();
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 8) {
    // ---- TMA producer -----------------------------------------------------------------------
    if (lane == 0) {
      mbar_expect_tx(&sm.q_full, kTileBytes);
      for (int x = 0; x < 2; ++x)
        tma_load_2d(smem_u32(sm.q) + (uint32_t)(x * kBoxBytes), &map_q, h * kD + x * 64,
                    start + q0, &sm.q_full);
      int issued = 0;
      for (int i = 0; i < tiles && !sm.error; ++i) {
        const int s = i % kRing;
        if (!mbar_wait(&sm.ring_empty[s], (uint32_t)(((i / kRing) & 1) ^ 1))) {
          sm.error = 1;
          break;
        }
        bool is_v;
        int kt;
        tile_of(i, n, is_v, kt);
        mbar_expect_tx(&sm.ring_full[s], kTileBytes);
        for (int x = 0; x < 2; ++x)
          tma_load_2d(smem_u32(sm.ring[s]) + (uint32_t)(x * kBoxBytes), is_v ? &map_v : &map_k,
                      hk * kD + x * 64, start + kt * kTile, &sm.ring_full[s]);
        ++issued;
      }
      // every copy issued must have landed before the CTA may leave (bounded)
      mbar_wait(&sm.q_full, 0);
      for (int i = issued - (issued < kRing ? issued : kRing); i < issued; ++i)
        mbar_wait(&sm.ring_full[i % kRing], (uint32_t)((i / kRing) & 1));
    }
  } else if (warp == 9) {
    // ---- MMA issuer -------------------------------------------------------------------------
    if (lane == 0) {
      uint32_t p_uses = 0;
      bool ok = mbar_wait(&sm.q_full, 0);
      const uint32_t q_addr = smem_u32(sm.q);
      for (int i = 0; i < tiles && ok && !sm.error; ++i) {
        const int s = i % kRing;
        bool is_v;
        int kt;
        tile_of(i, n, is_v, kt);
        if (!mbar_wait(&sm.ring_full[s], (uint32_t)((i / kRing) & 1))) {
          ok = false;
          break;
        }
        const uint32_t t_addr = smem_u32(sm.ring[s]);
        if (!is_v) {
          // S(kt) = Q K^T into buffer kt & 1, once the softmax has read that buffer's last use
          const int bf = kt & 1;
          if (!mbar_wait(&sm.s_read[bf], (uint32_t)(((kt >> 1) & 1) ^ 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_s = tmem + kColS + (uint32_t)(128 * bf);
#pragma unroll
          for (int k = 0; k < kD / 16; ++k) {
            const uint32_t off = (uint32_t)((k >> 2) * kBoxBytes + (k & 3) * 32);
            mma_ss(d_s, desc_k(q_addr + off), desc_k(t_addr + off), kIdescS, k != 0);
          }
          mma_commit(&sm.ring_empty[s]);
          mma_commit(&sm.s_full[bf]);
        } else {
          // O += P V once the softmax has written P
          if (!mbar_wait(&sm.p_full, p_uses & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int j = 0; j < kTile / 16; ++j)
            mma_ts(tmem + kColO, tmem + kColP + (uint32_t)(8 * j),
                   desc_mn(t_addr + (uint32_t)(j * 2048)), kIdescO, (kt | j) != 0);
          mma_commit(&sm.ring_empty[s]);
          mma_commit(&sm.p_free);
          ++p_uses;
        }
      }
      if (!ok) sm.error = 1;
      mma_commit(&sm.o_full);
      mma_commit(&sm.mma_done);
      if (!mbar_wait(&sm.mma_done, 0)) sm.error = 1;  // no MMA in flight before TMEM is freed
    }
  } else {
    // ---- softmax (warps 0-7): thread = query row = TMEM lane, two threads a row -------------
    const int quarter = warp & 3, hcol = warp >> 2;  // lane quarter; key / column half
    const int row = quarter * 32 + lane;
    const int qi = q0 + row;  // query index within the sequence
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    uint32_t p_uses = 0;
    bool go = true;  // false after a wait gave up: the loop still runs to the end (bounded)
    float m = -CUDART_INF_F, l = 0.f;
    for (int kt = 0; kt < n; ++kt) {
      const int bf = kt & 1;
      const uint32_t s_col = kColS + (uint32_t)(128 * bf);
      go = __all_sync(0xffffffffu, go && mbar_wait(&sm.s_full[bf], (uint32_t)((kt >> 1) & 1)));
      tc_fence_after();
      // no masked key for any row of this CTA in a tile below the diagonal and inside the
      // sequence (warp-uniform): the tile maximum is that of the raw scores, scaled once
      const bool full = kt < qt && (kt + 1) * kTile <= len;
      float mt = -CUDART_INF_F;
#pragma unroll 1
      for (int c = 0; c < kTile / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(lane_base + s_col + (uint32_t)(32 * c), v);
        if (full) {
#pragma unroll
          for (int e = 0; e < 32; ++e) mt = fmaxf(mt, __uint_as_float(v[e]));
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int key = kt * kTile + 32 * c + e;
            if (key <= qi && key < len) mt = fmaxf(mt, __uint_as_float(v[e]) * a.scale_log2);
          }
        }
      }
      if (full) mt *= a.scale_log2;
      // P must not be overwritten before the last P V has read it
      go = __all_sync(0xffffffffu, go && mbar_wait(&sm.p_free, (p_uses & 1) ^ 1));
      tc_fence_after();
      // a new reference maximum only when this tile's exceeds the kept one by 2^kRescaleAt
      // (the first tile sets it); this thread's half of O is rescaled in TMEM to match
      const bool move = kt == 0 || mt > m + kRescaleAt;
      const float m_new = move ? fmaxf(m, mt) : m;
      const float f = (kt == 0 || !move) ? 1.f : ex2a(m - m_new);
      if (kt > 0 && __any_sync(0xffffffffu, move)) {
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          const uint32_t o_col = kColO + (uint32_t)(64 * hcol + 32 * c);
          uint32_t v[32];
          tmem_ld32(lane_base + o_col, v);
          uint32_t lo[16], hi[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            lo[e] = __float_as_uint(__uint_as_float(v[e]) * f);
            hi[e] = __float_as_uint(__uint_as_float(v[16 + e]) * f);
          }
          tmem_st16(lane_base + o_col, lo);
          tmem_st16(lane_base + o_col + 16, hi);
        }
      }
      l *= f;
      m = m_new;
      // P = 2^(s - m) for this thread's 64 keys (fp16 into TMEM), the half-row sum from the
      // same fp32 values
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        const int kc = 64 * hcol + 32 * c;  // first key of the chunk within the tile
        uint32_t v[32], pk[16];
        tmem_ld32(lane_base + s_col + (uint32_t)kc, v);
        if (full) {
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float p0 = ex2a(__uint_as_float(v[e]) * a.scale_log2 - m);
            const float p1 = ex2a(__uint_as_float(v[e + 1]) * a.scale_log2 - m);
            l += p0 + p1;
            pk[e >> 1] = pack_half2(p0, p1);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const int key = kt * kTile + kc + e;
            const float p0 = (key <= qi && key < len)
                                 ? ex2a(__uint_as_float(v[e]) * a.scale_log2 - m) : 0.f;
            const float p1 = (key + 1 <= qi && key + 1 < len)
                                 ? ex2a(__uint_as_float(v[e + 1]) * a.scale_log2 - m) : 0.f;
            l += p0 + p1;
            pk[e >> 1] = pack_half2(p0, p1);
          }
        }
        tmem_st16(lane_base + kColP + (uint32_t)(kc >> 1), pk);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.s_read[bf]);  // this S buffer may take tile kt + 2
        mbar_arrive(&sm.p_full);      // P (and a rescaled O) ready for P V
      }
      ++p_uses;
    }
    // epilogue: the two half-row sums added (first half + second half, in that order), O / l
    // (fp16) and the base-2 log-sum-exp, rows of this sequence only
    go = __all_sync(0xffffffffu, go && mbar_wait(&sm.o_full, 0));
    sm.l_pair[hcol][row] = l;
    asm volatile("bar.sync 1, 256;" ::: "memory");  // the 8 softmax warps, all of them here
    tc_fence_after();
    const float total = sm.l_pair[0][row] + sm.l_pair[1][row];
    const float inv = 1.f / total;
    uint16_t *dst =
        a.out + ((int64_t)start + qi) * ((int64_t)a.n_heads * kD) + (int64_t)h * kD + 64 * hcol;
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t v[32];
      tmem_ld32(lane_base + kColO + (uint32_t)(64 * hcol + 32 * c), v);
      if (go && qi < len) {
        uint4 *d4 = reinterpret_cast<uint4 *>(dst + 32 * c);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          d4[q] = make_uint4(
              pack_half2(__uint_as_float(v[8 * q]) * inv, __uint_as_float(v[8 * q + 1]) * inv),
              pack_half2(__uint_as_float(v[8 * q + 2]) * inv, __uint_as_float(v[8 * q + 3]) * inv),
              pack_half2(__uint_as_float(v[8 * q + 4]) * inv, __uint_as_float(v[8 * q + 5]) * inv),
              pack_half2(__uint_as_float(v[8 * q + 6]) * inv, __uint_as_float(v[8 * q + 7]) * inv));
      }
    }
    if (go && qi < len && hcol == 0) a.lse[(int64_t)h * a.total + start + qi] = m + __log2f(total);
    if (!go && lane == 0) sm.error = 1;
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && sm.error) atomicAdd(&g_wait_timeouts, 1u);
  if (warp == 9) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// ---- host ---------------------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// token-major fp16 [rows, cols] -> boxes of 128 rows x 64 columns, 128-byte swizzle
int make_map(CUtensorMap *map, const void *base, int64_t rows, int64_t cols) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr)
    return set_error(TB_EDEVICE, "attn_varlen_fwd_tc: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)kTile};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                        strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(TB_EINVAL, "attn_varlen_fwd_tc: tensor map encode failed (%d)", (int)r);
  return TB_OK;
}

}  // namespace

TB_REGISTER_TIMEOUT_READER(attention_tc)

}  // namespace tb

using namespace tb;

extern "C" int tb_attn_varlen_fwd_tc(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                                     const int32_t *cu_seqlens, uint16_t *out, float *lse,
                                     int64_t batch, int64_t total, int64_t max_len,
                                     int32_t n_heads, int32_t n_kv, int32_t head_dim, float scale,
                                     void *stream) {
  if (head_dim != kD)
    return set_error(TB_EINVAL, "attn_varlen_fwd_tc: head_dim %d (the kernel takes %d)", head_dim,
                     kD);
  if (batch < 0 || total < 0 || max_len < 0 || n_heads < 1 || n_kv < 1 || n_heads % n_kv ||
      batch > 65535 || n_heads > 65535 || (max_len + kTile - 1) / kTile > 65535 ||
      total > (1LL << 31))
    return set_error(TB_EINVAL, "attn_varlen_fwd_tc: batch %lld total %lld max_len %lld heads "
                     "%d/%d", (long long)batch, (long long)total, (long long)max_len, n_heads, n_kv);
  if (!q || !k || !v || !cu_seqlens || !out || !lse)
    return set_error(TB_EINVAL, "attn_varlen_fwd_tc: q, k, v, cu_seqlens, out, lse required");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16))
    return set_error(TB_EALIGN, "attn_varlen_fwd_tc: q, k, v, out must be 16-byte aligned");
  if (batch == 0 || total == 0 || max_len == 0) return TB_OK;
  int dev = 0, major = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return set_error(TB_EDEVICE, "attn_varlen_fwd_tc: needs an sm_100 GPU");
  CUtensorMap mq, mk, mv;
  int rc = make_map(&mq, q, total, (int64_t)n_heads * kD);
  if (rc == TB_OK) rc = make_map(&mk, k, total, (int64_t)n_kv * kD);
  if (rc == TB_OK) rc = make_map(&mv, v, total, (int64_t)n_kv * kD);
  if (rc != TB_OK) return rc;
  const size_t smem = sizeof(Smem) + 1024;
  if (cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return check_launch("attn_varlen_fwd_tc attribute");
  TcArgs a{cu_seqlens, out, lse, total, n_heads, n_kv, scale * 1.4426950408889634f};
  const dim3 grid((unsigned)n_heads, (unsigned)batch, (unsigned)((max_len + kTile - 1) / kTile));
  attn_fwd_tc_kernel<<<grid, kThreads, smem, as_stream(stream)>>>(mq, mk, mv, a);
  note_launch();
  return check_launch("attn_varlen_fwd_tc");
}
