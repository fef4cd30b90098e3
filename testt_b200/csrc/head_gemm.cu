// Vocabulary head on the 5th-generation tensor cores: logits = h . W^T with tcgen05.mma (TMEM
// accumulators, TMA-fed shared-memory operands) and the online-softmax partial statistics of
// each (row, 256-column vocabulary tile) computed in the epilogue, so the logits never have to be
// read back for sweep 1 of the reference's head kernel (solution/head.py:54-72).
//
// One persistent CTA per SM, warp-specialised:
//   warp 0       TMA producer: per K block of 64, a 128x64 tile of h and a 256x64 tile of W
//                (fp16, K-major, 128-byte swizzle) into a 4-stage shared-memory ring
//   warp 1       MMA issuer: 4 x tcgen05.mma.kind::f16 (M128 N256 K16) per stage into one of two
//                TMEM accumulators (2 x 256 fp32 columns, double-buffered across tiles)
//   warps 2..5   epilogue: tcgen05.ld of the tile's rows (warp w reads TMEM lanes 32*(w%4)..),
//                logits rounded to fp16 exactly as the reference's fp16 GEMM output, then per row
//                (max, sum e, sum e z, first argmax, z[target]) -> part[row][vtile], and
//                optionally the fp16 logits for the dlogits / dh pass.
// tb_head_merge then merges the vocabulary tiles into lse, entropy, loss and the argmax hit.
// Tiles are ordered so concurrent CTAs share vocabulary tiles (W streamed from HBM about once).
// Every mbarrier wait is bounded (mbar_wait); a role that gives up leaves its loop, all roles
// meet at the final barrier and TMEM is always deallocated. No multicast is used.
#include <cuda.h>

#include <math_constants.h>

#include "common.cuh"

namespace tb {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;   // tile; kBK fp16 = 128 bytes = one swizzle row
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK * 2;          // 16 KB
constexpr int kBBytes = kBN * kBK * 2;          // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;  // 48 KB
constexpr int kThreads = 192;                   // 6 warps
constexpr int kTmemCols = 2 * kBN;              // two fp32 accumulators
constexpr int kPartFields = 6;

// M=128, N=256, A=B=f16 (K-major), D=f32: the kind::f16 instruction descriptor
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);

// Each epilogue warp's staging tile for the kept logits: 32 rows of 32 fp16 values in 80-byte
// rows (the 8 rows a quarter-warp touches at once fall in distinct 16-byte bank groups).
constexpr int kOutLd = 40;  // halves per staged row

struct Smem {
  alignas(1024) uint8_t stage[kStages][kStageBytes];  // A then B per stage (1024-aligned atoms)
  alignas(16) uint16_t out_stage[4][32 * kOutLd];
  uint64_t full[kStages], empty[kStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  volatile int error;  // a role gave up waiting: every role leaves its loop
};

// K-major, 128-byte-swizzle operand descriptor: start address, LBO 1 (ignored for swizzled
// K-major), SBO 1024 bytes between 8-row atoms, version 1 (sm_100), layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3fff);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma_f16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(kIdesc), "r"(acc)
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

constexpr float kLog2e = 1.4426950408889634f;

// 2^x on the MUFU (PTX ex2.approx); e^x is computed as 2^(x log2 e)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One row's online state over one 256-column vocabulary tile, built 32 columns at a time.
struct RowTile {
  float m, s, dz;  // running max; sum of e = exp(z - m); sum of e z
  float zt, pm;    // the target's logit; max of the target chunk's columns before the target
  int fm_chunk;    // column offset of the first chunk that reached the running max
  bool found;      // the target lies in this tile
  bool first;      // ... and is the tile's first maximum
};

// Folds 32 fp16 logits (packed in pairs, column c.. of the tile) into the state. The chunk max
// is taken on the packed halves; the argmax is not tracked per element: only whether the
// target is the tile's first maximum matters (tb_head_merge compares the winning index with
// the target), which needs the target's chunk alone (t_off = target - tile column 0, or
// negative when the target is elsewhere). kFull false: only the first nvalid columns exist.
template <bool kFull>
__device__ __forceinline__ void fold_chunk(RowTile &st, uint32_t (&h)[16], int c, int nvalid,
                                           int t_off) {
  if (!kFull) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {  // columns past the vocabulary: -inf (no max, e = 0)
      if (2 * j >= nvalid) h[j] = (h[j] & 0xffff0000u) | 0xfc00u;
      if (2 * j + 1 >= nvalid) h[j] = (h[j] & 0x0000ffffu) | 0xfc000000u;
    }
  }
  __half2 v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    v[j] = __hmax2(*reinterpret_cast<const __half2 *>(&h[j]),
                   *reinterpret_cast<const __half2 *>(&h[j + 8]));
#pragma unroll
  for (int w = 4; w > 0; w >>= 1)
#pragma unroll
    for (int j = 0; j < w; ++j) v[j] = __hmax2(v[j], v[j + w]);
  const float lm = fmaxf(__low2float(v[0]), __high2float(v[0]));
  if (lm > st.m) {
    const float sc = ex2_approx((st.m - lm) * kLog2e);  // 0 while m is -inf
    st.s *= sc;
    st.dz *= sc;
    st.m = lm;
    st.fm_chunk = c;
  }
  const float ml = st.m * kLog2e;
  float s0 = 0.f, s1 = 0.f, d0 = 0.f, d1 = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float2 z = __half22float2(*reinterpret_cast<const __half2 *>(&h[j]));
    const float e0 = ex2_approx(fmaf(z.x, kLog2e, -ml));
    const float e1 = ex2_approx(fmaf(z.y, kLog2e, -ml));
    s0 += e0;
    s1 += e1;
    d0 = fmaf(e0, kFull || 2 * j < nvalid ? z.x : 0.f, d0);
    d1 = fmaf(e1, kFull || 2 * j + 1 < nvalid ? z.y : 0.f, d1);
  }
  st.s += s0 + s1;
  st.dz += d0 + d1;
  const int o = t_off - c;
  if ((unsigned)o < 32u) {  // the target's chunk (one per labelled row)
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float2 z = __half22float2(*reinterpret_cast<const __half2 *>(&h[j]));
      if (2 * j < o) st.pm = fmaxf(st.pm, z.x);
      if (2 * j == o) st.zt = z.x;
      if (2 * j + 1 < o) st.pm = fmaxf(st.pm, z.y);
      if (2 * j + 1 == o) st.zt = z.y;
    }
    st.found = true;
  }
}

struct HeadArgs {
  const int64_t *targets;
  uint16_t *logits;  // optional fp16 [logits_rows, vocab] output
  float *part;       // [rows, n_vtiles, 6]
  int64_t *part_idx; // [rows, n_vtiles]
  int rows, logits_rows, vocab, k_blocks, m_tiles, v_tiles;
};

// The epilogue of one tile for one row (one thread): reads the row's 256 fp32 accumulator
// columns from TMEM (taddr: this warp's lane quarter and the accumulator), rounds them to fp16
// as the reference's fp16 GEMM output, optionally stores them (kept rows) and returns the
// tile's state. Every thread of the warp calls it (tcgen05.ld is warp-wide). The kept logits of
// a 32-column chunk go through the warp's staging tile `buf`: each lane writes its row there,
// then every store instruction writes 8 rows x 64 contiguous bytes (one lane a row would make
// each 16-byte store land in 32 different rows: 806 against 661 us for config 4's head GEMM
// with and without the kept logits).
__device__ __forceinline__ RowTile tile_rows(const HeadArgs &args, uint32_t taddr, int row,
                                             bool live, int64_t target, int col0,
                                             uint16_t *buf) {
  RowTile st{-CUDART_INF_F, 0.f, 0.f, 0.f, -CUDART_INF_F, -1, false, false};
  const int64_t dt = target - col0;
  const int t_off = (dt >= 0 && dt < kBN) ? (int)dt : -1024;
  const bool keep = live && args.logits != nullptr && row < args.logits_rows;
  const bool warp_keeps = __any_sync(0xffffffffu, keep);
  const int lane = threadIdx.x & 31, row0 = row - lane;
#pragma unroll 1
  for (int c = 0; c < kBN; c += 32) {
    const int nvalid = min(32, args.vocab - (col0 + c));
    if (nvalid <= 0) break;  // warp-uniform: the rest of the tile is past the vocabulary
    uint32_t r[32];
    tmem_ld32(taddr + (uint32_t)c, r);
    uint32_t h[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const __half2 hh = __floats2half2_rn(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
      h[j] = *reinterpret_cast<const uint32_t *>(&hh);
    }
    if (warp_keeps && nvalid == 32 && (args.vocab & 7) == 0) {  // warp-uniform
      uint4 *mine = reinterpret_cast<uint4 *>(buf + lane * kOutLd);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        mine[q] = make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
      __syncwarp();
#pragma unroll
      for (int it = 0; it < 4; ++it) {  // rows it*8 + (lane % 8), 16-byte part lane / 8
        const int r = it * 8 + (lane & 7), part = lane >> 3;
        const uint4 v = *reinterpret_cast<const uint4 *>(buf + r * kOutLd + part * 8);
        if (row0 + r < args.logits_rows)
          *reinterpret_cast<uint4 *>(args.logits + (int64_t)(row0 + r) * args.vocab + col0 + c +
                                     part * 8) = v;
      }
      __syncwarp();  // the tile is rewritten by the next chunk
    } else if (keep) {
      uint16_t *dst = args.logits + (int64_t)row * args.vocab + col0 + c;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < nvalid) dst[i] = (uint16_t)(h[i / 2] >> (16 * (i & 1)));
    }
    if (nvalid == 32)
      fold_chunk<true>(st, h, c, 32, t_off);
    else
      fold_chunk<false>(st, h, c, nvalid, t_off);
  }
  // the target is the tile's first maximum: it reaches the max, its chunk is the first chunk
  // that does, and no column of that chunk before it does
  st.first = st.found && st.zt == st.m && st.fm_chunk == (t_off & ~31) && st.pm < st.m;
  return st;
}

// part[row][vt] = (m, s, dz, m, zt, found) and an index that tb_head_merge orders tiles by and
// that equals the target exactly when the target is this tile's first maximum (any other
// column of the tile otherwise)
__device__ __forceinline__ void store_partial(const HeadArgs &args, int row, int vt, int col0,
                                              int64_t target, const RowTile &st) {
  const int64_t at = (int64_t)row * args.v_tiles + vt;
  float *out = args.part + at * kPartFields;
  out[0] = st.m;
  out[1] = st.s;
  out[2] = st.dz;
  out[3] = st.m;
  out[4] = st.found ? st.zt : 0.f;
  out[5] = st.found ? 1.f : 0.f;
  args.part_idx[at] = st.first ? target : (int64_t)col0 + (target == col0 ? 1 : 0);
}

__global__ void __launch_bounds__(kThreads, 1)
    head_logits_stats(const __grid_constant__ CUtensorMap map_h,
                      const __grid_constant__ CUtensorMap map_w, const HeadArgs args) {
  extern __shared__ uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                        ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tiles = (int64_t)args.m_tiles * args.v_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sm.acc_full[a], 1);
      mbar_init(&sm.acc_empty[a], 4);
    }
    mbar_init(&sm.mma_done, 1);
    sm.error = 0;
    mbar_init_fence();
  }
  if (warp == 1) {  // TMEM: two 256-column fp32 accumulators
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

  if (warp == 0) {
    // ---- TMA producer -------------------------------------------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      for (int64_t t = blockIdx.x; t < tiles && !sm.error; t += gridDim.x) {
        const int mt = (int)(t % args.m_tiles), vt = (int)(t / args.m_tiles);
        for (int kb = 0; kb < args.k_blocks; ++kb) {
          if (!mbar_wait(&sm.empty[stage], phase ^ 1)) {
            sm.error = 1;
            break;
          }
          mbar_expect_tx(&sm.full[stage], kStageBytes);
          tma_load_2d(sm.stage[stage], &map_h, kb * kBK, mt * kBM, &sm.full[stage]);
          tma_load_2d(sm.stage[stage] + kABytes, &map_w, kb * kBK, vt * kBN, &sm.full[stage]);
          ++issued;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // every copy issued must have landed before the CTA may leave (bounded)
      for (int s = 0; s < kStages && s < (int)issued; ++s) {
        if (stage == 0) {
          stage = kStages;
          phase ^= 1;
        }
        --stage;
        mbar_wait(&sm.full[stage], phase);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ---------------------------------------------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t it = 0;
      for (int64_t t = blockIdx.x; t < tiles && !sm.error; t += gridDim.x, ++it) {
        const int acc = (int)(it & 1);
        const uint32_t acc_phase = (uint32_t)((it >> 1) & 1);
        if (!mbar_wait(&sm.acc_empty[acc], acc_phase ^ 1)) {
          sm.error = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * kBN);
        for (int kb = 0; kb < args.k_blocks; ++kb) {
          if (!mbar_wait(&sm.full[stage], phase)) {
            sm.error = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sm.stage[stage]);
          const uint32_t b0 = a0 + kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)  // K = 16 per MMA: 32 bytes along the swizzled row
            mma_f16(d, smem_desc(a0 + k * 32), smem_desc(b0 + k * 32), (kb | k) != 0);
          mma_commit(&sm.empty[stage]);  // the stage is free once these MMAs have read it
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        mma_commit(&sm.acc_full[acc]);  // the accumulator is ready once all its MMAs are done
      }
      mma_commit(&sm.mma_done);
      mbar_wait(&sm.mma_done, 0);  // no MMA in flight before TMEM is released
    }
  } else {
    // ---- epilogue: 4 warps, thread = one row of the tile ----------------------------------
    const int quarter = warp & 3;                // TMEM lanes 32*quarter .. 32*quarter+31
    const int row_in_tile = quarter * 32 + lane;
    int64_t it = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
      const int acc = (int)(it & 1);
      const uint32_t acc_phase = (uint32_t)((it >> 1) & 1);
      const int ok = mbar_wait(&sm.acc_full[acc], acc_phase) ? 1 : 0;
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) sm.error = 1;
        break;
      }
      tc_fence_after();
      const int mt = (int)(t % args.m_tiles), vt = (int)(t / args.m_tiles);
      const int row = mt * kBM + row_in_tile;
      const bool live = row < args.rows;
      const int64_t target = live ? __ldg(args.targets + row) : -1;
      const int col0 = vt * kBN;
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * kBN);
      const RowTile st = tile_rows(args, taddr, row, live, target, col0, sm.out_stage[quarter]);
      // the accumulator may be overwritten once every epilogue warp has read it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[acc]);
      if (live) store_partial(args, row, vt, col0, target, st);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && sm.error) atomicAdd(&g_wait_timeouts, 1u);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// ---- 2-SM version: a CTA pair computes a 256x256 tile with tcgen05.mma.cta_group::2 ------------
// CTA rank r of the pair loads rows [256*mt + 128 r, +128) of h and rows [256*vt + 128 r, +128) of
// W into its own shared memory (6 stages of 32 KB); both CTAs' TMA loads complete on the leader's
// (rank 0) full barrier, which the leader alone arms for 64 KB. The leader's MMA thread issues
// M256 N256 K16 MMAs: each CTA's TMEM receives its own 128 rows x 256 columns (double-buffered).
// Commits are multicast to the same barrier in both CTAs (stage empty, accumulator full); each
// CTA's epilogue drains its own TMEM and arrives on the leader's accumulator-empty barrier
// (8 arrivals). Operand reuse is 131 FLOP per byte loaded, against 87 for the 1-SM tile.
constexpr int kStages2 = 6;
constexpr int kA2Bytes = 128 * kBK * 2;            // 16 KB: this CTA's rows of h
constexpr int kB2Bytes = 128 * kBK * 2;            // 16 KB: this CTA's half of the W tile
constexpr int kStage2Bytes = kA2Bytes + kB2Bytes;  // 32 KB
constexpr uint32_t kPeerMask = 0xFEFFFFFFu;        // shared::cluster address -> rank 0 of the pair
constexpr uint32_t kIdesc2 =
    (1u << 4) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);

struct Smem2 {
  alignas(1024) uint8_t stage[kStages2][kStage2Bytes];
  alignas(16) uint16_t out_stage[4][32 * kOutLd];
  uint64_t full[kStages2], empty[kStages2];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  volatile int error;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, int c0, int c1,
                                                 uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar) & kPeerMask)
      : "memory");
}

__device__ __forceinline__ void mma_f16_pair(uint32_t tmem, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(kIdesc2), "r"(acc)
      : "memory");
}

// arrive on the barrier at this offset in both CTAs of the pair once prior MMAs complete
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\t"
      "mov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], m;\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_leader(uint64_t *bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                   smem_u32(bar) & kPeerMask)
               : "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    head_logits_stats_2sm(const __grid_constant__ CUtensorMap map_h,
                          const __grid_constant__ CUtensorMap map_w, const HeadArgs args) {
  extern __shared__ uint8_t smem_raw[];
  Smem2 &sm = *reinterpret_cast<Smem2 *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                          ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int64_t pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int m_tiles2 = (args.rows + 255) / 256;
  const int64_t tiles = (int64_t)m_tiles2 * args.v_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sm.acc_full[a], 1);
      mbar_init(&sm.acc_empty[a], 8);  // 4 epilogue warps in each CTA of the pair
    }
    mbar_init(&sm.mma_done, 1);
    sm.error = 0;
    mbar_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, issued = 0;
      for (int64_t t = pair; t < tiles && !sm.error; t += pairs) {
        const int mt = (int)(t % m_tiles2), vt = (int)(t / m_tiles2);
        for (int kb = 0; kb < args.k_blocks; ++kb) {
          if (!mbar_wait(&sm.empty[stage], phase ^ 1)) {
            sm.error = 1;
            break;
          }
          if (leader) mbar_expect_tx(&sm.full[stage], 2 * kStage2Bytes);
          tma_load_2d_pair(sm.stage[stage], &map_h, kb * kBK, mt * 256 + (int)rank * 128,
                           &sm.full[stage]);
          tma_load_2d_pair(sm.stage[stage] + kA2Bytes, &map_w, kb * kBK,
                           vt * kBN + (int)rank * 128, &sm.full[stage]);
          ++issued;
          if (++stage == kStages2) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // this CTA's copies have landed once the stages it filled are freed again (bounded)
      for (int s = 0; s < kStages2 && s < (int)issued; ++s) {
        if (stage == 0) {
          stage = kStages2;
          phase ^= 1;
        }
        --stage;
        mbar_wait(&sm.empty[stage], phase);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t it = 0;
      for (int64_t t = pair; t < tiles && !sm.error; t += pairs, ++it) {
        const int acc = (int)(it & 1);
        const uint32_t acc_phase = (uint32_t)((it >> 1) & 1);
        if (!mbar_wait(&sm.acc_empty[acc], acc_phase ^ 1)) {
          sm.error = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * kBN);
        for (int kb = 0; kb < args.k_blocks; ++kb) {
          if (!mbar_wait(&sm.full[stage], phase)) {
            sm.error = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sm.stage[stage]);
          const uint32_t b0 = a0 + kA2Bytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_f16_pair(d, smem_desc(a0 + k * 32), smem_desc(b0 + k * 32), (kb | k) != 0);
          mma_commit_pair(&sm.empty[stage]);
          if (++stage == kStages2) {
            stage = 0;
            phase ^= 1;
          }
        }
        mma_commit_pair(&sm.acc_full[acc]);
      }
      asm volatile(
          "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
              smem_u32(&sm.mma_done))
          : "memory");
      mbar_wait(&sm.mma_done, 0);
    }
  } else {
    const int quarter = warp & 3;
    const int row_in_tile = (int)rank * 128 + quarter * 32 + lane;
    int64_t it = 0;
    for (int64_t t = pair; t < tiles; t += pairs, ++it) {
      const int acc = (int)(it & 1);
      const uint32_t acc_phase = (uint32_t)((it >> 1) & 1);
      const int ok = mbar_wait(&sm.acc_full[acc], acc_phase) ? 1 : 0;
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) sm.error = 1;
        break;
      }
      tc_fence_after();
      const int mt = (int)(t % m_tiles2), vt = (int)(t / m_tiles2);
      const int row = mt * 256 + row_in_tile;
      const bool live = row < args.rows;
      const int64_t target = live ? __ldg(args.targets + row) : -1;
      const int col0 = vt * kBN;
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * kBN);
      const RowTile st = tile_rows(args, taddr, row, live, target, col0, sm.out_stage[quarter]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_leader(&sm.acc_empty[acc]);
      if (live) store_partial(args, row, vt, col0, target, st);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while its pair may still reach its shared memory
  if (threadIdx.x == 0 && sm.error) atomicAdd(&g_wait_timeouts, 1u);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// ---- host: TMA descriptors through the driver entry point (no libcuda link) ---------------

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

// 2-D fp16 row-major [rows, cols] -> box [box_rows, 64] with 128-byte swizzle
int make_map(CUtensorMap *map, const void *base, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return set_error(TB_EDEVICE, "head: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                        strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TB_EINVAL, "head: tensor map encode failed (%d)", (int)r);
  return TB_OK;
}

// 0: automatic, 1: the 1-SM kernel, 2: the 2-SM kernel (process-wide; tb_head_gemm_variant)
int g_head_variant = 0;
constexpr bool kAutoTwoSm = false;

}  // namespace

TB_REGISTER_TIMEOUT_READER(head_gemm)

}  // namespace tb

using namespace tb;

extern "C" int tb_head_logits_stats(const uint16_t *hidden, const uint16_t *weight,
                                    const int64_t *targets, uint16_t *logits, int64_t logits_rows,
                                    float *part, int64_t *part_idx, int64_t rows, int64_t vocab,
                                    int64_t hidden_dim, void *stream) {
  if (rows < 0 || vocab <= 0 || hidden_dim <= 0)
    return set_error(TB_EINVAL, "head_logits_stats: rows %lld vocab %lld hidden %lld",
                     (long long)rows, (long long)vocab, (long long)hidden_dim);
  if (rows == 0) return TB_OK;
  if (!hidden || !weight || !targets || !part || !part_idx)
    return set_error(TB_EINVAL, "head_logits_stats: hidden, weight, targets, part, part_idx required");
  if (hidden_dim % kBK != 0)
    return set_error(TB_EINVAL, "head_logits_stats: hidden size %lld is not a multiple of %d",
                     (long long)hidden_dim, kBK);
  if (!aligned(hidden, 16) || !aligned(weight, 16) || (logits && !aligned(logits, 16)))
    return set_error(TB_EALIGN, "head_logits_stats: 16-byte aligned buffers are required");
  if (rows > (1LL << 30) || vocab > (1LL << 30))
    return set_error(TB_EINVAL, "head_logits_stats: sizes too large");
  int dev = 0, major = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return set_error(TB_EDEVICE, "head_logits_stats: needs an sm_100 GPU");
  CUtensorMap map_h, map_w;
  int rc = make_map(&map_h, hidden, rows, hidden_dim, kBM);
  if (rc == TB_OK) rc = make_map(&map_w, weight, vocab, hidden_dim, kBN);
  if (rc != TB_OK) return rc;
  HeadArgs a;
  a.targets = targets;
  a.logits = logits;
  a.part = part;
  a.part_idx = part_idx;
  a.rows = (int)rows;
  a.logits_rows = logits ? (int)(logits_rows < rows ? logits_rows : rows) : 0;
  a.vocab = (int)vocab;
  a.k_blocks = (int)(hidden_dim / kBK);
  a.m_tiles = (int)((rows + kBM - 1) / kBM);
  a.v_tiles = (int)((vocab + kBN - 1) / kBN);
  const int variant = g_head_variant;
  const bool two_sm = variant == 2 || (variant == 0 && kAutoTwoSm && rows > kBM);
  if (two_sm) {
    CUtensorMap map_h2, map_w2;  // boxes of 128 rows for both operands
    rc = make_map(&map_h2, hidden, rows, hidden_dim, 128);
    if (rc == TB_OK) rc = make_map(&map_w2, weight, vocab, hidden_dim, 128);
    if (rc != TB_OK) return rc;
    const size_t smem2 = sizeof(Smem2) + 1024;
    if (cudaFuncSetAttribute(head_logits_stats_2sm, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem2) != cudaSuccess)
      return check_launch("head_logits_stats_2sm attribute");
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem2;
    cfg.stream = as_stream(stream);
    cfg.gridDim = dim3(2 * (unsigned)sm_count());
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, head_logits_stats_2sm, &cfg) != cudaSuccess ||
        clusters < 1)
      return check_launch("head_logits_stats_2sm occupancy");
    const int64_t tiles2 = (int64_t)((rows + 255) / 256) * a.v_tiles;
    const int64_t pairs = tiles2 < clusters ? tiles2 : clusters;
    head_logits_stats_2sm<<<(unsigned)(2 * pairs), kThreads, smem2, as_stream(stream)>>>(
        map_h2, map_w2, a);
    note_launch();
    return check_launch("head_logits_stats_2sm");
  }
  const size_t smem = sizeof(Smem) + 1024;
  if (cudaFuncSetAttribute(head_logits_stats, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return check_launch("head_logits_stats attribute");
  const int64_t tiles = (int64_t)a.m_tiles * a.v_tiles;
  const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
  head_logits_stats<<<grid, kThreads, smem, as_stream(stream)>>>(map_h, map_w, a);
  note_launch();
  return check_launch("head_logits_stats");
}

extern "C" int tb_head_gemm_variant(int32_t variant) {
  if (variant < 0 || variant > 2)
    return set_error(TB_EINVAL, "head_gemm_variant: %d (0 auto, 1 one-SM, 2 two-SM)", variant);
  g_head_variant = variant;
  return TB_OK;
}
