// The head's hidden-state gradient on the 5th-generation tensor cores, with the logits gradient
// formed in the operand producer (reference: solution/head.py:73-76 writes dlogits in place,
// then :113 dh_chunk = dlogits[:lab] @ W with cuBLAS):
//
//   dl[r, c] = fp16((e^(z[r, c] - lse[r]) - [col_offset + c == target[r]]) * grad_scale)
//   dh[r, :] = sum_c dl[r, c] W[c, :]                       (fp32 accumulation in TMEM)
//
// z are the fp16 logits the logits GEMM kept (tb_head_logits_stats), so dl is never written to
// memory: the 2-byte read of z replaces the read + write + read of the in-place dlogits pass.
// dl is computed exactly as tb_head_dlogits computes it (same instructions, same rounding).
//
// MMA: D[r, n] = A[r, :] . B[n, :] with A = dl (128 rows x 32 vocabulary columns per stage,
// K-major, 64-byte swizzle, written by the producer warps) and B = W (32 vocabulary rows x 512
// hidden columns, MN-major: W's hidden columns are contiguous, 128-byte swizzle, 8 TMA boxes of
// 64 x 32), two M128 N256 K16 instructions per 16 columns into two TMEM accumulators (512
// columns, all of TMEM).
//
// Work split: CTA (s, t, g) computes the fp32 partial of row tile t and hidden group g (512
// columns) over the s-th of S contiguous vocabulary ranges (S = SMs / (row tiles x groups), at
// least 1). Block indices put the group fastest, then the row tile, then the range: the CTAs
// that read the same logits tile (same row tile and range, every group) and the CTAs that read
// the same W block (same group and range, every row tile) run side by side at the same pace, so
// logits and W come from HBM about once and are served to the others from L2. Each CTA writes
// one partial (128 x 512) to the caller's workspace; head_dh_reduce sums the S partials of each
// output element in range order (deterministic), maps rows and writes fp32 or fp16.
//
// CTA (10 warps):
//   warp 0      TMA producer: per vocabulary block the 128 x 32 fp16 logits tile (no swizzle)
//               and W's 32 x 512 block (one 3-D copy), into a 4-stage ring
//   warp 1      TMEM allocation (512 columns) and the MMA issuer
//   warps 2..9  producers of A: logits tile -> dl (fp16, swizzled) for the MMA, 16 rows a warp;
//               at the end the epilogue: TMEM -> fp32 partial in the workspace (warps w and
//               w + 4 share TMEM lane quarter w % 4, each reading half the columns)
// Every mbarrier wait is bounded (mbar_wait); a role that gives up sets the CTA's error flag and
// leaves its loop, every role meets at the final barrier and TMEM is always released. No
// multicast is used.
#include <cuda.h>

#include "common.cuh"

namespace tb {
namespace {

constexpr int kBM = 128;       // dh rows per tile
constexpr int kBN = 512;       // hidden columns per group (two N = 256 accumulators)
constexpr int kHalf = 256;
constexpr int kBK = 32;        // vocabulary columns per unit: 64 bytes of fp16
constexpr int kStages = 4;
constexpr int kRawBytes = kBM * kBK * 2;   // 8 KB: fp16 logits, 64-byte rows
constexpr int kABytes = kBM * kBK * 2;     // 8 KB: fp16 dl, K-major, 64-byte swizzle
constexpr int kBBytes = kBK * kBN * 2;     // 32 KB: W block, MN-major, 128-byte swizzle
constexpr int kBoxBytes = kBK * 64 * 2;    // one TMA box of W: 32 rows x 64 columns
constexpr int kThreads = 320;
constexpr int kProducers = 256;            // warps 2..9
constexpr int kTmemCols = 512;
constexpr int kMaxGroups = 16;             // hidden <= 8192
constexpr float kLog2e = 1.4426950408889634f;

// M = 128, N = 256, A = B = f16, D = f32, A K-major, B MN-major (bit 16)
constexpr uint32_t kIdesc = (1u << 4) | (1u << 16) | ((uint32_t)(kHalf >> 3) << 17) |
                            ((uint32_t)(kBM >> 4) << 24);

struct Smem {
  alignas(1024) uint8_t b[kStages][kBBytes];
  alignas(1024) uint8_t a[kStages][kABytes];
  alignas(128) uint8_t raw[kStages][kRawBytes];
  uint64_t full_raw[kStages], full_b[kStages], full_a[kStages], empty[kStages];
  uint64_t acc_full, mma_done;
  uint32_t tmem_base;
  volatile int error;
};

struct DhArgs {
  const int64_t *targets;   // [rows], global column of the label (IGNORE_INDEX: none)
  const float *lse;         // [rows]
  float *ws;                // partials [S][m_tiles][groups][128][512] fp32, block order
  int rows, cols, hidden;
  int64_t col_offset;
  float grad_scale;
  int m_tiles, groups;      // row tiles of 128, hidden groups of 512
  int splits, kblocks;      // S vocabulary ranges; vocabulary blocks of 32
};

// K-major operand, 64-byte swizzle: SBO 512 bytes between 8-row atoms (LBO unused), sm_100
__device__ __forceinline__ uint64_t desc_a(uint32_t addr) {
  uint64_t d = (uint64_t)((addr >> 4) & 0x3fff);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(512 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)4 << 61;
  return d;
}

// MN-major operand, 128-byte swizzle: LBO 4096 bytes between 64-column blocks (one TMA box),
// SBO 1024 bytes between 8-row groups along K, sm_100
__device__ __forceinline__ uint64_t desc_b(uint32_t addr) {
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

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
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

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Vocabulary blocks [lo, hi) of range s of S.
__device__ __host__ __forceinline__ void kb_range(int s, int splits, int kblocks, int &lo,
                                                  int &hi) {
  lo = (int)((int64_t)kblocks * s / splits);
  hi = (int)((int64_t)kblocks * (s + 1) / splits);
}

__global__ void __launch_bounds__(kThreads, 1)
    head_dh_kernel(const __grid_constant__ CUtensorMap map_z,
                   const __grid_constant__ CUtensorMap map_w, const __grid_constant__ DhArgs args) {
  extern __shared__ uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                        ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = (int)(blockIdx.x % args.groups);
  const int mt = (int)((blockIdx.x / args.groups) % args.m_tiles);
  const int sp = (int)(blockIdx.x / (args.groups * args.m_tiles));
  int k0, k1;
  kb_range(sp, args.splits, args.kblocks, k0, k1);
  const int n = k1 - k0;
  const int width = min(kBN, args.hidden - g * kBN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full_raw[s], 1);
      mbar_init(&sm.full_b[s], 1);
      mbar_init(&sm.full_a[s], kProducers);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.acc_full, 1);
    mbar_init(&sm.mma_done, 1);
    sm.error = 0;
    mbar_init_fence();
  }
  if (warp == 1) {
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
    // ---- TMA producer ---------------------------------------------------------------------
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < n && !sm.error; ++i) {
        const int s = i % kStages;
        const uint32_t parity = (uint32_t)((i / kStages) & 1);
        if (!mbar_wait(&sm.empty[s], parity ^ 1)) {
          sm.error = 1;
          break;
        }
        const int kb = k0 + i;
        mbar_expect_tx(&sm.full_raw[s], kRawBytes);
        tma_load_2d(smem_u32(sm.raw[s]), &map_z, kb * kBK, mt * kBM, &sm.full_raw[s]);
        // W's 32 x 512 block as one copy: 8 column blocks of 64 (the map's third dimension),
        // each a 32 x 64 MN-major atom column; blocks past the hidden size are zero-filled
        mbar_expect_tx(&sm.full_b[s], (uint32_t)kBBytes);
        tma_load_3d(smem_u32(sm.b[s]), &map_w, 0, kb * kBK, g * (kBN / 64), &sm.full_b[s]);
        ++issued;
      }
      // every copy issued must have landed before the CTA may leave (bounded)
      for (int i = issued - (issued < kStages ? issued : kStages); i < issued; ++i) {
        mbar_wait(&sm.full_raw[i % kStages], (uint32_t)((i / kStages) & 1));
        mbar_wait(&sm.full_b[i % kStages], (uint32_t)((i / kStages) & 1));
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer -------------------------------------------------------------------------
    if (lane == 0) {
      const int halves = width / kHalf;
      for (int i = 0; i < n && !sm.error; ++i) {
        const int s = i % kStages;
        const uint32_t parity = (uint32_t)((i / kStages) & 1);
        if (!mbar_wait(&sm.full_b[s], parity) || !mbar_wait(&sm.full_a[s], parity)) {
          sm.error = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sm.a[s]), b0 = smem_u32(sm.b[s]);
        for (int h = 0; h < halves; ++h)
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)  // K = 16 per MMA: 32 bytes along A's rows,
                                              // two 8-row groups (2 KB) down B
            mma_f16(tmem + (uint32_t)(h * kHalf), desc_a(a0 + k * 32),
                    desc_b(b0 + (uint32_t)(h * 4 * kBoxBytes) + k * 2048),
                    (i != 0 || k != 0) ? 1u : 0u);
        mma_commit(&sm.empty[s]);  // the stage is free once these MMAs have read it
      }
      mma_commit(&sm.acc_full);
      mma_commit(&sm.mma_done);
      if (!mbar_wait(&sm.mma_done, 0)) sm.error = 1;  // no MMA in flight before TMEM is released
    }
  } else {
    // ---- producers of A (dl), then the epilogue ------------------------------------------------
    const int tw = warp - 2, quarter = warp & 3;
    const int c = lane & 3;  // 16-byte chunk (8 columns) of the 64-byte rows
    float nl[2];
    int64_t target[2];
    bool live[2];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int r = mt * kBM + tw * 16 + p * 8 + (lane >> 2);
      live[p] = r < args.rows;
      target[p] = live[p] ? __ldg(args.targets + r) : -100;
      if (target[p] == -100) live[p] = false;
      nl[p] = live[p] ? -__ldg(args.lse + r) * kLog2e : 0.f;
    }
    bool go = true;
    for (int i = 0; i < n && !sm.error; ++i) {
      const int kb = k0 + i;
      const int s = i % kStages;
      if (!mbar_wait(&sm.full_raw[s], (uint32_t)((i / kStages) & 1))) {
        sm.error = 1;
        go = false;
        break;
      }
      const uint32_t raw = smem_u32(sm.raw[s]), a = smem_u32(sm.a[s]);
      const int c0 = kb * kBK + c * 8;  // local column of this thread's 8 values
      const int64_t gc0 = args.col_offset + c0;
      const bool ragged = kb * kBK + kBK > args.cols;  // the last block of a partial slab
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int row = tw * 16 + p * 8 + (lane >> 2);
        uint4 zv;
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(zv.x), "=r"(zv.y), "=r"(zv.z), "=r"(zv.w)
                     : "r"(raw + (uint32_t)(row * 64 + c * 16)));
        const uint32_t w[4] = {zv.x, zv.y, zv.z, zv.w};
        // the label's position among this thread's 8 columns, -1 if elsewhere
        const int tl = (uint64_t)(target[p] - gc0) < 8u ? (int)(target[p] - gc0) : -1;
        float g8[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 z = unpack_half2(w[e]);
          g8[2 * e] = ex2f(fmaf(z.x, kLog2e, nl[p]));
          g8[2 * e + 1] = ex2f(fmaf(z.y, kLog2e, nl[p]));
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float v = g8[e];
          if (e == tl) v -= 1.f;
          v *= args.grad_scale;
          g8[e] = live[p] ? v : 0.f;
        }
        if (ragged) {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (c0 + e >= args.cols) g8[e] = 0.f;
        }
        const uint32_t dst = a + (uint32_t)(row * 64) + ((uint32_t)(c ^ ((row >> 1) & 3)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst),
                     "r"(pack_half2(g8[0], g8[1])), "r"(pack_half2(g8[2], g8[3])),
                     "r"(pack_half2(g8[4], g8[5])), "r"(pack_half2(g8[6], g8[7]))
                     : "memory");
      }
      fence_proxy_async();  // the generic-proxy stores, visible to the tensor core
      mbar_arrive(&sm.full_a[s]);
    }
    // epilogue: this warp's lane quarter, columns [half * 256, half * 256 + 256) of the group
    const int half = tw >> 2;
    if (go && n > 0 && half * kHalf < width) {
      const int ok = mbar_wait(&sm.acc_full, 0) ? 1 : 0;
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) sm.error = 1;
      } else {
        tc_fence_after();
        const int rr = quarter * 32 + lane;
        float *dst = args.ws + ((int64_t)blockIdx.x * kBM + rr) * kBN + half * kHalf;
        for (int col = 0; col < kHalf; col += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * kHalf + col), v);
          float4 *d4 = reinterpret_cast<float4 *>(dst + col);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            d4[q] = make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
        }
      }
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

struct ReduceArgs {
  const float *ws;
  int rows, hidden, m_tiles, groups, splits;
  const int64_t *out_rows;             // nullable: dh row r -> output row out_rows[r]
  void *out;
  int64_t ld_out;
  int out_fp32, accumulate;
};

// out[row(r), c] (+)= sum over the vocabulary ranges s (in order) of their partial for (r, c).
__global__ void __launch_bounds__(256) head_dh_reduce(const __grid_constant__ ReduceArgs a) {
  pdl_wait();
  pdl_release();
  const int64_t vecs = (int64_t)a.rows * (a.hidden / 4);
  const int64_t split_stride = (int64_t)a.m_tiles * a.groups * kBM * kBN;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < vecs;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(v / (a.hidden / 4));
    const int col = (int)(v - (int64_t)r * (a.hidden / 4)) * 4;
    const int mt = r / kBM, rr = r % kBM, g = col / kBN, cc = col % kBN;
    const float *p = a.ws + (((int64_t)mt * a.groups + g) * kBM + rr) * kBN + cc;
    float4 acc = *reinterpret_cast<const float4 *>(p);
    for (int s = 1; s < a.splits; ++s) {
      const float4 q = *reinterpret_cast<const float4 *>(p + s * split_stride);
      acc.x = __fadd_rn(acc.x, q.x);
      acc.y = __fadd_rn(acc.y, q.y);
      acc.z = __fadd_rn(acc.z, q.z);
      acc.w = __fadd_rn(acc.w, q.w);
    }
    const int64_t orow = a.out_rows ? __ldg(a.out_rows + r) : r;
    if (a.out_fp32) {
      float4 *o = reinterpret_cast<float4 *>(static_cast<float *>(a.out) + orow * a.ld_out + col);
      if (a.accumulate) {
        const float4 old = *o;
        acc.x = __fadd_rn(old.x, acc.x);
        acc.y = __fadd_rn(old.y, acc.y);
        acc.z = __fadd_rn(old.z, acc.z);
        acc.w = __fadd_rn(old.w, acc.w);
      }
      *o = acc;
    } else {
      uint2 *o = reinterpret_cast<uint2 *>(static_cast<uint16_t *>(a.out) + orow * a.ld_out + col);
      *o = make_uint2(pack_half2(acc.x, acc.y), pack_half2(acc.z, acc.w));
    }
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

// fp16 row-major [rows, cols] (row stride ld elements) -> box [box_rows, box_cols]
int make_map(CUtensorMap *map, const void *base, int64_t rows, int64_t cols, int64_t ld,
             int box_cols, int box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return set_error(TB_EDEVICE, "head_dh: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                        strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TB_EINVAL, "head_dh: tensor map encode failed (%d)", (int)r);
  return TB_OK;
}

// W fp16 [cols, hidden] (row-major) viewed as [hidden / 64][cols][64]: box [8][32][64], so one
// copy brings a 32 x 512 block as 8 consecutive 4 KB atom columns (128-byte swizzle)
int make_map_w(CUtensorMap *map, const void *base, int64_t cols, int64_t hidden) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return set_error(TB_EDEVICE, "head_dh: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {64, (cuuint64_t)cols, (cuuint64_t)(hidden / 64)};
  const cuuint64_t strides[2] = {(cuuint64_t)hidden * 2, 128};
  const cuuint32_t box[3] = {64, (cuuint32_t)kBK, (cuuint32_t)(kBN / 64)};
  const cuuint32_t estride[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims,
                        strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TB_EINVAL, "head_dh: W map encode failed (%d)", (int)r);
  return TB_OK;
}

struct Plan {
  int m_tiles, groups, splits, kblocks;
};

// S vocabulary ranges per (row tile, hidden group): as many as fill the SMs with one CTA each,
// at least 1, at most one per vocabulary block.
Plan make_plan(int64_t rows, int64_t cols, int64_t hidden, int sms) {
  Plan p{};
  p.m_tiles = (int)((rows + kBM - 1) / kBM);
  p.groups = (int)((hidden + kBN - 1) / kBN);
  p.kblocks = (int)((cols + kBK - 1) / kBK);
  int splits = sms / (p.m_tiles * p.groups);
  if (splits < 1) splits = 1;
  if (splits > p.kblocks) splits = p.kblocks;
  p.splits = splits;
  return p;
}

int64_t workspace_bytes(const Plan &p) {
  return (int64_t)p.splits * p.m_tiles * p.groups * kBM * kBN * 4;
}

}  // namespace

TB_REGISTER_TIMEOUT_READER(head_dh)

}  // namespace tb

using namespace tb;

static int dh_shape_error(int64_t rows, int64_t cols, int64_t hidden) {
  if (rows < 0 || rows > (1LL << 24) || cols <= 0 || cols > (1LL << 30))
    return set_error(TB_EINVAL, "head_dh: rows %lld cols %lld", (long long)rows, (long long)cols);
  if (hidden <= 0 || hidden % 256 != 0 || hidden > kMaxGroups * kBN)
    return set_error(TB_EINVAL, "head_dh: hidden size %lld (a multiple of 256, at most %d)",
                     (long long)hidden, kMaxGroups * kBN);
  return TB_OK;
}

extern "C" int64_t tb_head_dh_workspace(int64_t rows, int64_t cols, int64_t hidden_dim) {
  if (rows <= 0 || dh_shape_error(rows, cols, hidden_dim) != TB_OK) return 0;
  return workspace_bytes(make_plan(rows, cols, hidden_dim, sm_count()));
}

extern "C" int tb_head_dh(const uint16_t *logits, int64_t ld, const int64_t *targets,
                          const float *lse, int64_t rows, int64_t cols, int64_t col_offset,
                          float grad_scale, const uint16_t *weight, int64_t hidden_dim,
                          float *workspace, int64_t workspace_bytes_given, void *out,
                          int32_t out_fp32, const int64_t *out_rows, int64_t ld_out,
                          int32_t accumulate, void *stream) {
  int rc = dh_shape_error(rows, cols, hidden_dim);
  if (rc != TB_OK) return rc;
  if (rows == 0) return TB_OK;
  if (!logits || !targets || !lse || !weight || !workspace || !out)
    return set_error(TB_EINVAL, "head_dh: logits, targets, lse, weight, workspace, out required");
  if (ld < cols || ld % 8 != 0 || ld_out < hidden_dim || ld_out % 4 != 0)
    return set_error(TB_EINVAL, "head_dh: ld %lld (>= cols, a multiple of 8), ld_out %lld "
                     "(>= hidden, a multiple of 4)", (long long)ld, (long long)ld_out);
  if (accumulate && !out_fp32)
    return set_error(TB_EINVAL, "head_dh: accumulation needs the fp32 output");
  if (!aligned(logits, 16) || !aligned(weight, 16) || !aligned(workspace, 16) ||
      !aligned(out, out_fp32 ? 16 : 8))
    return set_error(TB_EALIGN, "head_dh: 16-byte aligned logits, weight, workspace and out");
  int dev = 0, major = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return set_error(TB_EDEVICE, "head_dh: needs an sm_100 GPU");
  const Plan p = make_plan(rows, cols, hidden_dim, sm_count());
  if (workspace_bytes_given < workspace_bytes(p))
    return set_error(TB_EINVAL, "head_dh: workspace of %lld bytes, %lld needed",
                     (long long)workspace_bytes_given, (long long)workspace_bytes(p));
  CUtensorMap map_z, map_w;
  rc = make_map(&map_z, logits, rows, cols, ld, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc == TB_OK)
    rc = make_map_w(&map_w, weight, cols, hidden_dim);
  if (rc != TB_OK) return rc;
  DhArgs a;
  a.targets = targets;
  a.lse = lse;
  a.ws = workspace;
  a.rows = (int)rows;
  a.cols = (int)cols;
  a.hidden = (int)hidden_dim;
  a.col_offset = col_offset;
  a.grad_scale = grad_scale;
  a.m_tiles = p.m_tiles;
  a.groups = p.groups;
  a.splits = p.splits;
  a.kblocks = p.kblocks;
  const size_t smem = sizeof(Smem) + 1024;
  if (cudaFuncSetAttribute(head_dh_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return check_launch("head_dh attribute");
  const int64_t grid = (int64_t)p.splits * p.m_tiles * p.groups;
  if (grid > 0x7fffffffLL) return set_error(TB_EINVAL, "head_dh: too many rows");
  head_dh_kernel<<<(unsigned)grid, kThreads, smem, as_stream(stream)>>>(map_z, map_w, a);
  note_launch();
  rc = check_launch("head_dh");
  if (rc != TB_OK) return rc;
  ReduceArgs r;
  r.ws = workspace;
  r.rows = (int)rows;
  r.hidden = (int)hidden_dim;
  r.m_tiles = p.m_tiles;
  r.groups = p.groups;
  r.splits = p.splits;
  r.out_rows = out_rows;
  r.out = out;
  r.ld_out = ld_out;
  r.out_fp32 = out_fp32;
  r.accumulate = accumulate;
  const int64_t vecs = rows * (hidden_dim / 4);
  int64_t blocks = (vecs + 255) / 256;
  const int cap = resident_blocks(head_dh_reduce, 256);
  if (blocks > cap) blocks = cap;
  return launch("head_dh_reduce", head_dh_reduce, dim3((unsigned)blocks), dim3(256), 0,
                as_stream(stream), r);
}
