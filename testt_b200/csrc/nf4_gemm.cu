// NF4-weight GEMMs on the 5th-generation tensor cores with the NF4 decode in the operand
// producer, so the fp16 copy of a frozen weight is never written to HBM:
//
//   forward   out[t, n] = fp16(sum_k x[t, k] W[n, k] (+ bias[n]))   FrozenNF4Linear.forward,
//                                                                 solution/nf4.py:115-118
//   backward  out[t, k] = fp16(sum_n dy[t, n] W[n, k])              FrozenNF4Linear.backward,
//                                                                 solution/nf4.py:121-127
//
// W is up to four NF4 weights stacked by rows (q|k|v, gate|up), each in bitsandbytes' packing
// (row-major, blocksize 64, element 2i in the high nibble of byte i) with its fp32 absmax per
// block given block-column-major, absmax_t[k / 64][row] (a nested state's absmax expanded once by
// the caller: code2[c] * absmax2[b / 256] + offset, each operation rounded on its own, as the
// unpack kernel does). Every decoded value is fp16(table[q] * absmax) rounded once: bit-identical
// to tb_nf4_unpack_*'s output, and the product differs from cuBLAS over the unpacked weight only
// by the order of the fp32 sums.
//
// The MMA computes D[m, t] = A[m, :] . B[t, :] with the tokens (x or dy, TMA, K-major, 128-byte
// swizzle) as B and a decoded 128-row tile of W as A:
//   forward   A[n][k] = W[n][k], K-major: 128 W rows x 64 columns per stage;
//   backward  A[k][n] = W[n][k], MN-major (bit 15 of the instruction descriptor): 64 W rows x
//             128 columns per stage, so W is decoded row by row in its natural order in both
//             directions (no transposition anywhere).
// A stage's 64-value row segments are decoded from packed bytes and absmax that TMA and a bulk
// copy brought into shared memory, into 128-byte swizzled rows at segment * 128 bytes (the same
// address for both operand majors).
//
// Persistent CTAs (one per SM) loop over work units (128-row tile, token group of <= 256, split of
// the reduction); token groups are the fastest-varying so the CTAs that decode the same packed
// tile run side by side and share it through L2. Warps:
//   warp 0       TMA producer: tokens tile, packed NF4 tile (TMA), absmax (bulk copy) per stage
//   warp 1       TMEM allocation (2 x 256 columns) and the MMA issuer
//   warps 2..5   epilogue (TMEM lane quarters), overlapping the next unit's main loop
//   warps 6..13  decoders: two threads per 64-value segment; each warp arrives once per stage
// A split reduction writes fp32 partials [split][token][row] to the caller's workspace, summed in
// split order by nf4_gemm_reduce (plain, + bias) or qkv_rope_finish (the q|k|v projection's
// bias, LoRA rows and rotary embedding, token-major outputs). tb_nf4_gemm_swiglu runs the MLP's
// GEMMs with SwiGLU in the epilogue: the gate|up forward (tile rows alternate gate and up
// features, so each feature's pair of values meets in neighbouring lanes of one warp) and down's
// dX (dact never written: the epilogue applies the in-place SwiGLU backward to gu).
// Every mbarrier wait is bounded (mbar_wait); a role that gives up sets the CTA's error flag and
// leaves its loop, every role meets at the final barrier and TMEM is always released. No
// multicast is used.
#include <cuda.h>

#include <cstddef>

#include "common.cuh"

namespace tb {
namespace {

constexpr int kMaxW = 4;
constexpr int kBM = 128;                        // A rows per tile
constexpr int kBK = 64;                         // reduction per stage: 128 bytes of fp16
constexpr int kStages = 4;
constexpr int kMaxBN = 256;                     // tokens per tile (the MMA's N)
constexpr int kABytes = kBM * kBK * 2;          // 16 KB decoded tile
constexpr int kBBytes = kMaxBN * kBK * 2;       // 32 KB tokens tile
constexpr int kPBytes = 4096;                   // packed NF4 of one stage (128 x 64 values)
constexpr int kSBytes = kBM * 4;                // their 128 absmax
constexpr int kDecoders = 256;                  // warps 6..13
constexpr int kThreads = 448;
constexpr int kTmemCols = 512;                  // two accumulators of 256 columns

struct Smem {
  alignas(1024) uint8_t b[kStages][kBBytes];
  alignas(1024) uint8_t a[kStages][kABytes];
  alignas(128) uint8_t packed[kStages][kPBytes];
  alignas(128) float scale[kStages][kBM];
  alignas(256) float table[kMaxW][64];          // 16 entries used; 256-byte aligned rows
  uint64_t full_b[kStages], full_p[kStages], full_a[kStages], empty[kStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  volatile int error;
};

// epilogue modes
constexpr int kPlain = 0, kPart = 1, kSwigluFwd = 2, kSwigluBwd = 3;

struct GemmArgs {
  const float *absmax_t[kMaxW];  // fp32 [k_dim / 64, rows_j]
  const float *table[kMaxW];
  int rows[kMaxW];
  int row_start[kMaxW + 1];  // first stacked W row of each weight; row_start[n_w] = all rows
  int n_w;
  int k_dim;                 // columns of W
  int a_rows;                // rows of the A operand: stacked rows forward, k_dim backward
  int red_blocks;            // reduction blocks of 64
  int tokens, bn, groups, splits, a_tiles;
  int trans;                 // backward: A = W^T, MN-major
  int mode;
  uint32_t idesc;
  const uint16_t *bias;      // kPlain forward only
  uint16_t *out;             // fp16 [tokens, a_rows] (row stride ld_out); kSwigluFwd: act
  int64_t ld_out;
  float *part;               // kPart: [splits, tokens, a_rows] fp32
  uint16_t *gu;              // SwiGLU modes: fp16 [tokens, 2 * inter] gate | up (row stride ld_gu)
  int64_t ld_gu;
  int inter;
};

// ---- tcgen05 / TMA helpers (PTX ISA: tcgen05.mma, cp.async.bulk.tensor) --------------------

// K-major, 128-byte-swizzle descriptor: start address, LBO 1 (unused for swizzled K-major), SBO
// 1024 bytes between 8-row atoms, version 1 (sm_100), SWIZZLE_128B.
__device__ __forceinline__ uint64_t desc_k(uint32_t addr) {
  uint64_t d = (uint64_t)((addr >> 4) & 0x3fff);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// MN-major, 128-byte-swizzle descriptor of the backward A tile: LBO 8192 bytes between the two
// 64-element halves of M (each 64 rows of K x 128 bytes), SBO 1024 bytes between 8-row groups
// along K.
__device__ __forceinline__ uint64_t desc_mn(uint32_t addr) {
  uint64_t d = (uint64_t)((addr >> 4) & 0x3fff);
  d |= (uint64_t)(8192 >> 4) << 16;
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

__device__ __forceinline__ void mma_f16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
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

__device__ __forceinline__ void st_shared16(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 ld_shared16(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// ---- NF4 decode ------------------------------------------------------------------------------

// Shared-memory address tab | byte b of x (tab 256-byte aligned), one byte permute.
__device__ __forceinline__ uint32_t table_addr(uint32_t x, uint32_t tab, int b) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(tab), "r"(0x7650u | (uint32_t)b));
  return r;
}

// fp16 of the 8 nibbles of `word` (high nibble of each byte first) times `scale`, packed in
// element order: each product rounded to fp32 (no FMA), then once to fp16.
__device__ __forceinline__ uint4 decode_word(uint32_t word, float scale, uint32_t tab) {
  const uint32_t lo4 = (word << 2) & 0x3c3c3c3cu;
  const uint32_t hi4 = (word >> 2) & 0x3c3c3c3cu;
  float f[8];
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    float hi, lo;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(hi) : "r"(table_addr(hi4, tab, b)));
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(lo) : "r"(table_addr(lo4, tab, b)));
    const float2 p = __fmul2_rn(make_float2(hi, lo), make_float2(scale, scale));
    f[2 * b] = p.x;
    f[2 * b + 1] = p.y;
  }
  return make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]), pack_half2(f[4], f[5]),
                    pack_half2(f[6], f[7]));
}

// the SwiGLU kernels' formulas (fast exponential and division, as the reference's lower to)
__device__ __forceinline__ float silu(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

__device__ __forceinline__ void swiglu_bwd_one(float dact, float g, float u, float &dg, float &du) {
  const float sig = __fdividef(1.0f, 1.0f + __expf(-g));
  const float d_silu = dact * u;
  dg = d_silu * sig * (1.0f + g * (1.0f - sig));
  du = dact * (g * sig);
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

__device__ __forceinline__ int weight_of(const GemmArgs &args, int row) {
  int j = 0;
#pragma unroll
  for (int i = 1; i < kMaxW; ++i)
    if (i < args.n_w && row >= args.row_start[i]) j = i;
  return j;
}

// A work unit: (A tile, split, token group), token groups fastest.
struct Unit {
  int a_tile, split, group, first, nblk;
};

__device__ __forceinline__ Unit unit_of(const GemmArgs &args, int u) {
  Unit r;
  r.group = u % args.groups;
  const int rest = u / args.groups;
  r.split = rest % args.splits;
  r.a_tile = rest / args.splits;
  const int q = args.red_blocks / args.splits, rem = args.red_blocks % args.splits;
  r.first = r.split * q + (r.split < rem ? r.split : rem);
  r.nblk = q + (r.split < rem ? 1 : 0);
  return r;
}

// The packed-weight tensor maps of the (up to four) weights, kernel parameters.
struct PackedMaps {
  const CUtensorMap *m[kMaxW];
  __device__ __forceinline__ const CUtensorMap *operator[](int j) const {
    return j == 0 ? m[0] : j == 1 ? m[1] : j == 2 ? m[2] : m[3];
  }
};

// Issues the copies of one stage of unit `un`, reduction block kb (absolute): the tokens tile,
// the weight's packed tile (TMA) and its absmax (bulk copies), all completing on the stage's
// barriers.
__device__ __forceinline__ void issue_stage(const GemmArgs &args, const PackedMaps &maps_p,
                                            const CUtensorMap *map_b, Smem &sm, int s,
                                            const Unit &un, int kb) {
  const int t0 = un.group * args.bn;
  mbar_expect_tx(&sm.full_b[s], (uint32_t)(args.bn * kBK * 2));
  tma_load_2d(smem_u32(sm.b[s]), map_b, kb * kBK, t0, &sm.full_b[s]);
  mbar_expect_tx(&sm.full_p[s], (uint32_t)(kPBytes + kSBytes));
  const uint32_t pk = smem_u32(sm.packed[s]);
  if (args.mode == kSwigluFwd) {
    // 64 gate rows, then the same 64 up rows
    const int f0 = un.a_tile * 64;
    for (int j = 0; j < 2; ++j) {
      tma_load_2d(pk + (uint32_t)(j * 2048), maps_p[j], kb * 32, f0, &sm.full_p[s]);
      bulk_load(&sm.scale[s][j * 64], args.absmax_t[j] + (int64_t)kb * args.rows[j] + f0, 256,
                &sm.full_p[s]);
    }
  } else if (!args.trans) {
    const int a0 = un.a_tile * kBM;
    const int j = weight_of(args, a0);
    const int lr = a0 - args.row_start[j];
    tma_load_2d(pk, maps_p[j], kb * 32, lr, &sm.full_p[s]);
    bulk_load(&sm.scale[s][0], args.absmax_t[j] + (int64_t)kb * args.rows[j] + lr, kSBytes,
              &sm.full_p[s]);
  } else {
    // W rows kb*64 .. (within one weight), columns a0 .. a0 + 127
    const int a0 = un.a_tile * kBM;
    const int n0 = kb * kBK;
    const int j = weight_of(args, n0);
    const int ln = n0 - args.row_start[j];
    tma_load_2d(pk, maps_p[j], a0 >> 1, ln, &sm.full_p[s]);
    for (int h = 0; h < 2; ++h)
      bulk_load(&sm.scale[s][h * 64],
                args.absmax_t[j] + (int64_t)((a0 >> 6) + h) * args.rows[j] + ln, 256,
                &sm.full_p[s]);
  }
}

template <int kMode, bool kTrans>
__global__ void __launch_bounds__(kThreads, 1)
    nf4_gemm_kernel(const __grid_constant__ CUtensorMap map_b,
                    const __grid_constant__ CUtensorMap map_p0,
                    const __grid_constant__ CUtensorMap map_p1,
                    const __grid_constant__ CUtensorMap map_p2,
                    const __grid_constant__ CUtensorMap map_p3,
                    const __grid_constant__ GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                        ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = args.a_tiles * args.splits * args.groups;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full_b[s], 1);
      mbar_init(&sm.full_p[s], 1);
      mbar_init(&sm.full_a[s], kDecoders / 32);
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
  for (int i = threadIdx.x; i < args.n_w * 16; i += kThreads)
    sm.table[i >> 4][i & 15] = __ldg(args.table[i >> 4] + (i & 15));
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
    // ---- TMA producer ----------------------------------------------------------------------
    if (lane == 0) {
      const PackedMaps maps = {{&map_p0, &map_p1, &map_p2, &map_p3}};
      uint32_t ctr = 0;
      for (int u = blockIdx.x; u < units && !sm.error; u += gridDim.x) {
        const Unit un = unit_of(args, u);
        for (int i = 0; i < un.nblk; ++i, ++ctr) {
          const int s = (int)(ctr % kStages);
          if (!mbar_wait(&sm.empty[s], ((ctr / kStages) & 1) ^ 1)) {
            sm.error = 1;
            break;
          }
          issue_stage(args, maps, &map_b, sm, s, un, un.first + i);
        }
      }
      // every copy issued must have landed before the CTA may leave (bounded)
      const uint32_t tail = ctr < kStages ? ctr : kStages;
      for (uint32_t c = ctr - tail; c < ctr; ++c) {
        mbar_wait(&sm.full_b[c % kStages], (c / kStages) & 1);
        mbar_wait(&sm.full_p[c % kStages], (c / kStages) & 1);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer -------------------------------------------------------------------------
    if (lane == 0) {
      uint32_t ctr = 0;
      int it = 0;
      for (int u = blockIdx.x; u < units && !sm.error; u += gridDim.x, ++it) {
        const Unit un = unit_of(args, u);
        const int acc = it & 1;
        if (!mbar_wait(&sm.acc_empty[acc], ((it >> 1) & 1) ^ 1)) {
          sm.error = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * 256);
        for (int i = 0; i < un.nblk; ++i, ++ctr) {
          const int s = (int)(ctr % kStages);
          const uint32_t parity = (ctr / kStages) & 1;
          if (!mbar_wait(&sm.full_b[s], parity) || !mbar_wait(&sm.full_a[s], parity)) {
            sm.error = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a_tile = smem_u32(sm.a[s]), b_tile = smem_u32(sm.b[s]);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // K = 16 per MMA: 32 bytes along a K-major row, 16 rows (2 KB) down an MN-major tile
            const uint64_t da = kTrans ? desc_mn(a_tile + k * 2048) : desc_k(a_tile + k * 32);
            mma_f16(d, da, desc_k(b_tile + k * 32), args.idesc, (i | k) != 0);
          }
          mma_commit(&sm.empty[s]);  // the stage is free once these MMAs have read it
        }
        if (sm.error) break;
        mma_commit(&sm.acc_full[acc]);
      }
      mma_commit(&sm.mma_done);
      if (!mbar_wait(&sm.mma_done, 0)) sm.error = 1;  // no MMA in flight before TMEM is freed
    }
  } else if (warp < 6) {
    // ---- epilogue: warp w reads TMEM lanes 32 * (w % 4) .. -----------------------------------
    const int quarter = warp & 3;
    const int r_in = quarter * 32 + lane;
    int it = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
      const Unit un = unit_of(args, u);
      const int acc = it & 1;
      const int ok = mbar_wait(&sm.acc_full[acc], (it >> 1) & 1) ? 1 : 0;
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) sm.error = 1;
        break;
      }
      tc_fence_after();
      const int t0 = un.group * args.bn;
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * 256);
      // the A row (output feature) of this lane
      int row;
      if (kMode == kSwigluFwd)
        row = un.a_tile * 64 + (r_in >> 1);   // feature; even lanes gate, odd lanes up
      else
        row = un.a_tile * kBM + r_in;
      float bias = 0.f;
      if (kMode == kPlain && args.bias != nullptr) bias = h2f(__ldg(args.bias + row));
      for (int c = 0; c < args.bn; c += 32) {
        const int tb = t0 + c;
        if (tb >= args.tokens) break;  // uniform across the warp
        uint32_t v[32];
        tmem_ld32(taddr + (uint32_t)c, v);
        // tokens of this column chunk that exist and belong to this unit's group
        const int ne = min(32, min(args.bn - c, args.tokens - tb));
        if (kMode == kPart) {
          float *p = args.part + ((int64_t)un.split * args.tokens + tb) * args.a_rows + row;
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (e < ne) p[(int64_t)e * args.a_rows] = __uint_as_float(v[e]);
        } else if (kMode == kPlain) {
          uint16_t *o = args.out + (int64_t)tb * args.ld_out + row;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            if (e >= ne) break;
            float x = __uint_as_float(v[e]);
            if (args.bias != nullptr) x = __fadd_rn(x, bias);
            o[(int64_t)e * args.ld_out] = f2h(x);
          }
        } else if (kMode == kSwigluFwd) {
          const bool up = lane & 1;
          uint16_t *g_out = args.gu + (int64_t)tb * args.ld_gu + (up ? args.inter : 0) + row;
          uint16_t *a_out = args.out + (int64_t)tb * args.ld_out + row;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const uint16_t x16 = f2h(__uint_as_float(v[e]));
            const uint16_t other = (uint16_t)__shfl_xor_sync(0xffffffffu, (uint32_t)x16, 1);
            if (e < ne) {
              g_out[(int64_t)e * args.ld_gu] = x16;
              if (!up) a_out[(int64_t)e * args.ld_out] = f2h(silu(h2f(x16)) * h2f(other));
            }
          }
        } else {  // kSwigluBwd: row = feature f of dact; gu's two halves updated in place
          uint16_t *pg = args.gu + (int64_t)tb * args.ld_gu + row;
#pragma unroll
          for (int h = 0; h < 32; h += 16) {
            uint16_t g16[16], u16[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const bool in = h + e < ne;
              g16[e] = in ? pg[(int64_t)(h + e) * args.ld_gu] : (uint16_t)0;
              u16[e] = in ? pg[(int64_t)(h + e) * args.ld_gu + args.inter] : (uint16_t)0;
            }
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              if (h + e >= ne) break;
              float dg, du;
              swiglu_bwd_one(h2f(f2h(__uint_as_float(v[h + e]))), h2f(g16[e]), h2f(u16[e]), dg,
                             du);
              pg[(int64_t)(h + e) * args.ld_gu] = f2h(dg);
              pg[(int64_t)(h + e) * args.ld_gu + args.inter] = f2h(du);
            }
          }
        }
      }
      // the accumulator may be overwritten once every epilogue warp has read it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[acc]);
    }
  } else {
    // ---- decoders: segment s = A row (64 values of one W row), two threads each -----------
    const int d = threadIdx.x - 192;  // 0 .. 255
    const int seg = d >> 1, half = d & 1;
    // packed bytes and absmax of the segment in the stage buffers
    uint32_t p_off;
    int s_idx, jseg;
    if (kMode == kSwigluFwd) {
      p_off = (uint32_t)((seg & 1) * 2048 + (seg >> 1) * 32);
      s_idx = (seg & 1) * 64 + (seg >> 1);
      jseg = seg & 1;
    } else if (kTrans) {
      p_off = (uint32_t)((seg & 63) * 64 + (seg >> 6) * 32);
      s_idx = seg;
      jseg = -1;
    } else {
      p_off = (uint32_t)(seg * 32);
      s_idx = seg;
      jseg = -1;
    }
    p_off += (uint32_t)(half * 16);
    const uint32_t a_row = (uint32_t)(seg * 128);
    const uint32_t swz = (uint32_t)(seg & 7);
    uint32_t ctr = 0;
    bool stop = false;
    // every exit decision is warp-uniform: the warp arrives once per stage, after __syncwarp
    for (int u = blockIdx.x; u < units && !stop; u += gridDim.x) {
      if (__any_sync(0xffffffffu, sm.error != 0)) break;
      const Unit un = unit_of(args, u);
      const int jt = kTrans ? 0 : (kMode == kSwigluFwd ? 0 : weight_of(args, un.a_tile * kBM));
      for (int i = 0; i < un.nblk; ++i, ++ctr) {
        const int s = (int)(ctr % kStages);
        if (!__all_sync(0xffffffffu, mbar_wait(&sm.full_p[s], (ctr / kStages) & 1))) {
          if (lane == 0) sm.error = 1;
          stop = true;
          break;
        }
        const int j = jseg >= 0 ? jseg : (kTrans ? weight_of(args, (un.first + i) * kBK) : jt);
        const uint32_t tab = smem_u32(&sm.table[j][0]);
        const uint4 w = ld_shared16(smem_u32(sm.packed[s]) + p_off);
        const float scale = sm.scale[s][s_idx];
        const uint32_t a_tile = smem_u32(sm.a[s]) + a_row;
        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t c = (uint32_t)(half * 4 + q);  // 16-byte chunk of the 128-byte row
          st_shared16(a_tile + ((c ^ swz) << 4), decode_word(words[q], scale, tab));
        }
        fence_proxy_async();  // this thread's generic-proxy stores, visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.full_a[s]);  // one arrival per decoder warp
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

// out[t, r] = fp16(sum over splits s in order of part[s, t, r] (+ bias[r])), 8 rows a thread.
__global__ void __launch_bounds__(256) nf4_gemm_reduce(const float *part, int splits,
                                                       int64_t tokens, int a_rows,
                                                       const uint16_t *bias, uint16_t *out,
                                                       int64_t ld_out) {
  pdl_wait();
  pdl_release();
  const int64_t vecs_per_row = a_rows >> 3;
  const int64_t total = tokens * vecs_per_row;
  const int64_t plane = tokens * (int64_t)a_rows;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = v / vecs_per_row;
    const int c = (int)(v - t * vecs_per_row) * 8;
    const float *p = part + t * a_rows + c;
    float acc[8], f[8];
    load8f(p, acc);
    for (int s = 1; s < splits; ++s) {
      load8f(p + s * plane, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = __fadd_rn(acc[e], f[e]);
    }
    if (bias != nullptr) {
      load8h(bias + c, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = __fadd_rn(acc[e], f[e]);
    }
    store8h(out + t * ld_out + c, acc);
  }
}

// The q|k|v projection finished from its fp32 partials: per token, head and rotation pair
// (p, p + 64): the splits summed in order, + bias, rounded to fp16 (the GEMM's output), + the
// LoRA rows (q, v), the rotary embedding (q, k), written token-major (what tb_rope_tokens_fwd
// writes from the GEMM's fp16 output).
struct QkvArgs {
  const float *part;
  int splits, tokens, a_rows;
  const uint16_t *bias, *lora_q, *lora_v;
  const float *cosv, *sinv;
  const int64_t *pos_idx;
  int seq, nh, nkv;
  uint16_t *q_out, *k_out, *v_out;
};

__global__ void __launch_bounds__(256) qkv_rope_finish(const __grid_constant__ QkvArgs a) {
  pdl_wait();
  pdl_release();
  constexpr int D = 128, H = 64;
  const int heads = a.nh + 2 * a.nkv;
  const int64_t total = (int64_t)a.tokens * heads * H;
  const int64_t plane = (int64_t)a.tokens * a.a_rows;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int pr = (int)(e % H);
    const int hr = (int)((e / H) % heads);
    const int tok = (int)(e / ((int64_t)H * heads));
    const float *p = a.part + (int64_t)tok * a.a_rows + hr * D + pr;
    float s1 = 0.f, s2 = 0.f;
    for (int s = 0; s < a.splits; ++s) {
      s1 = __fadd_rn(s1, __ldg(p + s * plane));
      s2 = __fadd_rn(s2, __ldg(p + s * plane + H));
    }
    if (a.bias != nullptr) {
      s1 = __fadd_rn(s1, h2f(__ldg(a.bias + hr * D + pr)));
      s2 = __fadd_rn(s2, h2f(__ldg(a.bias + hr * D + pr + H)));
    }
    float x1 = h2f(f2h(s1)), x2 = h2f(f2h(s2));  // the GEMM's fp16 output
    const uint16_t *lora = nullptr;
    uint16_t *dst;
    if (hr < a.nh) {
      lora = a.lora_q ? a.lora_q + ((int64_t)tok * a.nh + hr) * D : nullptr;
      dst = a.q_out + ((int64_t)tok * a.nh + hr) * D;
    } else if (hr < a.nh + a.nkv) {
      dst = a.k_out + ((int64_t)tok * a.nkv + hr - a.nh) * D;
    } else {
      const int hv = hr - a.nh - a.nkv;
      lora = a.lora_v ? a.lora_v + ((int64_t)tok * a.nkv + hv) * D : nullptr;
      dst = a.v_out + ((int64_t)tok * a.nkv + hv) * D;
    }
    if (lora != nullptr) {
      x1 = x1 + h2f(__ldg(lora + pr));
      x2 = x2 + h2f(__ldg(lora + pr + H));
    }
    float o1 = x1, o2 = x2;  // v: LoRA-added, not rotated
    if (hr < a.nh + a.nkv) {
      const int64_t pos = __ldg(a.pos_idx + tok);
      if (pos < 0) continue;  // no position: nothing written (as tb_rope_tokens_fwd)
      const int64_t t = pos % a.seq;
      const float c1 = __ldg(a.cosv + t * D + pr), c2 = __ldg(a.cosv + t * D + H + pr);
      const float n1 = __ldg(a.sinv + t * D + pr), n2 = __ldg(a.sinv + t * D + H + pr);
      o1 = x1 * c1 - x2 * n1;
      o2 = x2 * c2 + x1 * n2;
    }
    dst[pr] = f2h(o1);
    dst[pr + H] = f2h(o2);
  }
}

// ---- host -------------------------------------------------------------------------------------

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

// 2-D row-major [rows, cols] of `type` (elem bytes) with row stride ld elements -> box
// [box_rows, box_cols]
int make_map(CUtensorMap *map, CUtensorMapDataType type, int elem, const void *base, int64_t rows,
             int64_t cols, int64_t ld, int box_cols, int box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return set_error(TB_EDEVICE, "nf4_gemm: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * elem};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = fn(map, type, 2, const_cast<void *>(base), dims, strides, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TB_EINVAL, "nf4_gemm: tensor map encode failed (%d)", (int)r);
  return TB_OK;
}

// 0: automatic (the reduction split until the units fill the GPU), 1: never split
// (process-wide; tb_nf4_gemm_variant)
int g_variant = 0;

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

struct Plan {
  int bn, groups, splits;
};

// Tokens in groups of <= 256 (the MMA's N, a multiple of 16); the reduction split so that the
// units fill the GPU (at least 4 blocks of 64 a split, at most 16 splits).
Plan make_plan(int64_t tokens, int a_tiles, int red_blocks, int sms, bool may_split) {
  Plan p;
  const int64_t g0 = ceil_div(tokens, kMaxBN);
  p.bn = (int)(ceil_div(ceil_div(tokens, g0), 16) * 16);
  p.groups = (int)ceil_div(tokens, p.bn);
  const int64_t tiles = (int64_t)a_tiles * p.groups;
  int splits = 1;
  if (may_split && g_variant != 1 && tiles < sms) {
    splits = (int)(sms / tiles);
    const int most = red_blocks / 4 > 1 ? red_blocks / 4 : 1;
    if (splits > most) splits = most;
    if (splits > 16) splits = 16;
  }
  p.splits = splits;
  return p;
}

// Shared argument checks; fills the weight fields of `a`. Returns TB_OK or an error.
int gemm_args(int32_t transpose, int64_t tokens, int32_t n_weights, const uint8_t *const *packed,
              const float *const *absmax_t, const float *const *nf4_table, const int64_t *rows,
              int64_t k_dim, GemmArgs &a) {
  if (n_weights < 1 || n_weights > kMaxW || !packed || !absmax_t || !nf4_table || !rows)
    return set_error(TB_EINVAL, "nf4_gemm: 1..%d weights with packed, absmax, table, rows", kMaxW);
  if (tokens < 0 || tokens > (1LL << 24) || k_dim <= 0 || k_dim > (1LL << 20))
    return set_error(TB_EINVAL, "nf4_gemm: tokens %lld k_dim %lld", (long long)tokens,
                     (long long)k_dim);
  const int64_t k_align = transpose ? 128 : 64;
  if (k_dim % k_align != 0)
    return set_error(TB_EINVAL, "nf4_gemm: k_dim %lld is not a multiple of %lld",
                     (long long)k_dim, (long long)k_align);
  const int64_t r_align = transpose ? 64 : 128;
  int64_t total = 0;
  a.row_start[0] = 0;
  for (int j = 0; j < n_weights; ++j) {
    if (!packed[j] || !absmax_t[j] || !nf4_table[j])
      return set_error(TB_EINVAL, "nf4_gemm: weight %d has a missing pointer", j);
    if (rows[j] <= 0 || rows[j] % r_align != 0)
      return set_error(TB_EINVAL, "nf4_gemm: weight %d has %lld rows (a multiple of %lld needed)",
                       j, (long long)rows[j], (long long)r_align);
    if (!aligned(packed[j], 16) || !aligned(absmax_t[j], 16) || !aligned(nf4_table[j], 4))
      return set_error(TB_EALIGN, "nf4_gemm: weight %d is not aligned", j);
    a.absmax_t[j] = absmax_t[j];
    a.table[j] = nf4_table[j];
    a.rows[j] = (int)rows[j];
    total += rows[j];
    if (total > (1LL << 24)) return set_error(TB_EINVAL, "nf4_gemm: too many rows");
    a.row_start[j + 1] = (int)total;
  }
  for (int j = n_weights; j < kMaxW; ++j) {
    a.absmax_t[j] = nullptr;
    a.table[j] = nullptr;
    a.rows[j] = 0;
    a.row_start[j + 1] = (int)total;
  }
  a.n_w = n_weights;
  a.k_dim = (int)k_dim;
  a.trans = transpose ? 1 : 0;
  a.a_rows = transpose ? (int)k_dim : (int)total;
  a.red_blocks = transpose ? (int)(total / kBK) : (int)(k_dim / kBK);
  a.tokens = (int)tokens;
  a.bias = nullptr;
  a.out = nullptr;
  a.ld_out = 0;
  a.part = nullptr;
  a.gu = nullptr;
  a.ld_gu = 0;
  a.inter = 0;
  return TB_OK;
}

int device_ok(const char *what) {
  int dev = 0, major = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return set_error(TB_EDEVICE, "%s: needs an sm_100 GPU", what);
  return TB_OK;
}

// Launches the GEMM kernel of `mode` over the planned units. `packed` maps: one per weight,
// boxes of the mode's packed tile (forward 128 rows x 32 bytes, backward 64 rows x 64 bytes,
// SwiGLU forward 64 rows x 32 bytes).
int run_gemm(int mode, GemmArgs &a, const Plan &p, const uint16_t *tokens_in, int64_t ld_in,
             const uint8_t *const *packed, cudaStream_t stream, const char *what) {
  a.bn = p.bn;
  a.groups = p.groups;
  a.splits = p.splits;
  a.mode = mode;
  a.idesc = (1u << 4) | ((uint32_t)a.trans << 15) | ((uint32_t)(p.bn >> 3) << 17) |
            ((uint32_t)(kBM >> 4) << 24);
  const int64_t red_dim = (int64_t)a.red_blocks * kBK;
  CUtensorMap map_b, maps_p[kMaxW];
  int rc = make_map(&map_b, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, tokens_in, a.tokens, red_dim,
                    ld_in, kBK, p.bn, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != TB_OK) return rc;
  for (int j = 0; j < kMaxW; ++j) {
    const int jj = j < a.n_w ? j : 0;  // unused maps repeat the first weight's
    const int box_cols = a.trans ? 64 : 32;
    const int box_rows = mode == kSwigluFwd ? 64 : (a.trans ? 64 : 128);
    rc = make_map(&maps_p[j], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, packed[jj], a.rows[jj],
                  a.k_dim / 2, a.k_dim / 2, box_cols, box_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != TB_OK) return rc;
  }
  const int64_t units = (int64_t)a.a_tiles * p.splits * p.groups;
  if (units > 0x7fffffffLL) return set_error(TB_EINVAL, "%s: too many tiles", what);
  const int grid = (int)(units < sm_count() ? units : sm_count());
  const size_t smem = sizeof(Smem) + 1024;
  void (*kernel)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, GemmArgs) =
      nullptr;
  if (mode == kPlain)
    kernel = a.trans ? nf4_gemm_kernel<kPlain, true> : nf4_gemm_kernel<kPlain, false>;
  else if (mode == kPart)
    kernel = a.trans ? nf4_gemm_kernel<kPart, true> : nf4_gemm_kernel<kPart, false>;
  else if (mode == kSwigluFwd)
    kernel = nf4_gemm_kernel<kSwigluFwd, false>;
  else
    kernel = nf4_gemm_kernel<kSwigluBwd, true>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return check_launch(what);
  kernel<<<(unsigned)grid, kThreads, smem, stream>>>(map_b, maps_p[0], maps_p[1], maps_p[2],
                                                      maps_p[3], a);
  note_launch();
  return check_launch(what);
}

}  // namespace

TB_REGISTER_TIMEOUT_READER(nf4_gemm)

}  // namespace tb

using namespace tb;

extern "C" int64_t tb_nf4_gemm_workspace(int32_t transpose, int64_t tokens, int32_t n_weights,
                                         const int64_t *rows, int64_t k_dim) {
  if (n_weights < 1 || n_weights > kMaxW || rows == nullptr || tokens <= 0 || k_dim <= 0) return 0;
  int64_t total = 0;
  for (int j = 0; j < n_weights; ++j) total += rows[j];
  const int64_t a_rows = transpose ? k_dim : total;
  const int red_blocks = (int)((transpose ? total : k_dim) / kBK);
  const Plan p = make_plan(tokens, (int)(a_rows / kBM), red_blocks, sm_count(), true);
  return p.splits > 1 ? (int64_t)p.splits * tokens * a_rows * 4 : 0;
}

extern "C" int tb_nf4_gemm(int32_t transpose, const uint16_t *tokens_in, int64_t tokens,
                           int64_t ld_in, int32_t n_weights, const uint8_t *const *packed,
                           const float *const *absmax_t, const float *const *nf4_table,
                           const int64_t *rows, int64_t k_dim, const uint16_t *bias, uint16_t *out,
                           int64_t ld_out, float *workspace, int64_t workspace_bytes,
                           void *stream) {
  GemmArgs a;
  int rc = gemm_args(transpose, tokens, n_weights, packed, absmax_t, nf4_table, rows, k_dim, a);
  if (rc != TB_OK) return rc;
  if (tokens == 0) return TB_OK;
  const int64_t red_dim = (int64_t)a.red_blocks * kBK;
  if (!tokens_in || !out) return set_error(TB_EINVAL, "nf4_gemm: tokens_in and out required");
  if (transpose && bias) return set_error(TB_EINVAL, "nf4_gemm: no bias in the backward");
  if (ld_in < red_dim || ld_in % 8 != 0 || ld_out < a.a_rows || ld_out % 8 != 0)
    return set_error(TB_EINVAL, "nf4_gemm: ld_in %lld (>= %lld, multiple of 8) ld_out %lld "
                     "(>= %d, multiple of 8)", (long long)ld_in, (long long)red_dim,
                     (long long)ld_out, a.a_rows);
  if (!aligned(tokens_in, 16) || !aligned(out, 16) || (bias && !aligned(bias, 16)) ||
      (workspace && !aligned(workspace, 16)))
    return set_error(TB_EALIGN, "nf4_gemm: 16-byte aligned tokens_in, out, bias, workspace needed");
  rc = device_ok("nf4_gemm");
  if (rc != TB_OK) return rc;
  a.a_tiles = a.a_rows / kBM;
  Plan p = make_plan(tokens, a.a_tiles, a.red_blocks, sm_count(), true);
  if (p.splits > 1 && (workspace == nullptr ||
                       workspace_bytes < (int64_t)p.splits * tokens * a.a_rows * 4))
    p.splits = 1;  // no (or too small a) workspace: one unit per tile
  cudaStream_t st = as_stream(stream);
  if (p.splits == 1) {
    a.bias = bias;
    a.out = out;
    a.ld_out = ld_out;
    return run_gemm(kPlain, a, p, tokens_in, ld_in, packed, st, "nf4_gemm");
  }
  a.part = workspace;
  rc = run_gemm(kPart, a, p, tokens_in, ld_in, packed, st, "nf4_gemm");
  if (rc != TB_OK) return rc;
  const int64_t vecs = tokens * (a.a_rows / 8);
  const int64_t blocks64 = (vecs + 255) / 256;
  const int cap = resident_blocks(nf4_gemm_reduce, 256);
  const int blocks = (int)(blocks64 < cap ? blocks64 : cap);
  return launch("nf4_gemm_reduce", nf4_gemm_reduce, dim3((unsigned)blocks), dim3(256), 0, st,
                (const float *)workspace, p.splits, tokens, a.a_rows, bias, out, ld_out);
}

// The MLP's two NF4 GEMMs with SwiGLU in the epilogue (one split each):
//   forward  (backward == 0): weights (gate, up), each [inter, k_dim]; tokens_in = x
//            [tokens, k_dim]; writes gu = fp16(x [gate|up]^T) [tokens, 2 inter] (row stride
//            ld_gu) and act = fp16(silu(g) u) [tokens, inter] (row stride ld_act)
//   backward (backward == 1): weight (down,) [hidden, inter] (k_dim = inter); tokens_in = dy
//            [tokens, hidden]; dact = fp16(dy . W_down) stays in the epilogue, which overwrites
//            gu with d(gate|up) (act unused)
extern "C" int tb_nf4_gemm_swiglu(int32_t backward, const uint16_t *tokens_in, int64_t tokens,
                                  int64_t ld_in, int32_t n_weights, const uint8_t *const *packed,
                                  const float *const *absmax_t, const float *const *nf4_table,
                                  const int64_t *rows, int64_t k_dim, uint16_t *gu, int64_t ld_gu,
                                  uint16_t *act, int64_t ld_act, void *stream) {
  GemmArgs a;
  int rc = gemm_args(backward ? 1 : 0, tokens, n_weights, packed, absmax_t, nf4_table, rows,
                     k_dim, a);
  if (rc != TB_OK) return rc;
  const int64_t inter = backward ? k_dim : rows[0];
  if (backward ? n_weights != 1 : (n_weights != 2 || rows[1] != rows[0] || rows[0] % 64 != 0))
    return set_error(TB_EINVAL, "nf4_gemm_swiglu: (gate, up) of equal rows forward, (down,) "
                     "backward");
  if (tokens == 0) return TB_OK;
  const int64_t red_dim = (int64_t)a.red_blocks * kBK;
  if (!tokens_in || !gu || (!backward && !act))
    return set_error(TB_EINVAL, "nf4_gemm_swiglu: tokens_in, gu (and act forward) required");
  if (ld_in < red_dim || ld_in % 8 != 0 || ld_gu < 2 * inter || (!backward && ld_act < inter))
    return set_error(TB_EINVAL, "nf4_gemm_swiglu: ld_in %lld ld_gu %lld ld_act %lld",
                     (long long)ld_in, (long long)ld_gu, (long long)ld_act);
  if (!aligned(tokens_in, 16) || !aligned(gu, 2) || (act && !aligned(act, 2)))
    return set_error(TB_EALIGN, "nf4_gemm_swiglu: misaligned buffer");
  rc = device_ok("nf4_gemm_swiglu");
  if (rc != TB_OK) return rc;
  // forward tiles hold 64 features of each weight (rows alternate gate, up); backward tiles
  // 128 features of dact
  a.a_tiles = backward ? (int)(inter / kBM) : (int)(inter / 64);
  const Plan p = make_plan(tokens, a.a_tiles, a.red_blocks, sm_count(), false);
  a.out = act;
  a.ld_out = ld_act;
  a.gu = gu;
  a.ld_gu = ld_gu;
  a.inter = (int)inter;
  return run_gemm(backward ? kSwigluBwd : kSwigluFwd, a, p, tokens_in, ld_in, packed,
                  as_stream(stream), "nf4_gemm_swiglu");
}

static int qkv_rows(int32_t n_heads, int32_t n_kv, int64_t (&rows)[3]) {
  if (n_heads <= 0 || n_kv <= 0 || n_heads % n_kv != 0)
    return set_error(TB_EINVAL, "nf4_gemm_qkv_rope: heads %d kv %d", n_heads, n_kv);
  rows[0] = (int64_t)n_heads * kBM;
  rows[1] = rows[2] = (int64_t)n_kv * kBM;
  return TB_OK;
}

extern "C" int64_t tb_nf4_gemm_qkv_rope_workspace(int64_t tokens, int32_t n_heads, int32_t n_kv,
                                                  int64_t k_dim) {
  int64_t rows[3];
  if (tokens <= 0 || k_dim <= 0 || k_dim % kBK != 0 || qkv_rows(n_heads, n_kv, rows) != TB_OK)
    return 0;
  const int64_t a_rows = rows[0] + rows[1] + rows[2];
  const Plan p = make_plan(tokens, (int)(a_rows / kBM), (int)(k_dim / kBK), sm_count(), true);
  return (int64_t)p.splits * tokens * a_rows * 4;
}

// The q|k|v projection with its bias, the LoRA rows and the rotary embedding: weights (q, k, v) =
// [n_heads * 128, k_dim], [n_kv * 128, k_dim] twice; x [tokens, k_dim] (row stride ld_x); out q
// [tokens, n_heads, 128], k, v [tokens, n_kv, 128] (token-major, contiguous) = what
// tb_rope_tokens_fwd writes from the GEMM's fp16 output (solution/rope.py:24-75 with the padded
// scatter replaced by token-major rows). lora_q / lora_v fp16 or NULL; cos, sin fp32 [seq, 128];
// pos_idx int64 padded positions (t = pos % seq). The GEMM's fp32 partials go to `workspace`
// (tb_nf4_gemm_qkv_rope_workspace bytes).
extern "C" int tb_nf4_gemm_qkv_rope(const uint16_t *x, int64_t tokens, int64_t ld_x,
                                    const uint8_t *const *packed, const float *const *absmax_t,
                                    const float *const *nf4_table, int64_t k_dim,
                                    const uint16_t *bias, const uint16_t *lora_q,
                                    const uint16_t *lora_v, const float *cos, const float *sin,
                                    const int64_t *pos_idx, int64_t seq, int32_t n_heads,
                                    int32_t n_kv, uint16_t *q, uint16_t *k, uint16_t *v,
                                    float *workspace, int64_t workspace_bytes, void *stream) {
  int64_t rows[3];
  int rc = qkv_rows(n_heads, n_kv, rows);
  if (rc != TB_OK) return rc;
  if (seq <= 0) return set_error(TB_EINVAL, "nf4_gemm_qkv_rope: seq %lld", (long long)seq);
  GemmArgs a;
  rc = gemm_args(0, tokens, 3, packed, absmax_t, nf4_table, rows, k_dim, a);
  if (rc != TB_OK) return rc;
  if (tokens == 0) return TB_OK;
  if (!x || !cos || !sin || !pos_idx || !q || !k || !v || !workspace)
    return set_error(TB_EINVAL, "nf4_gemm_qkv_rope: x, cos, sin, pos_idx, q, k, v, workspace "
                     "required");
  if (ld_x < k_dim || ld_x % 8 != 0 || !aligned(x, 16) || !aligned(workspace, 16))
    return set_error(TB_EINVAL, "nf4_gemm_qkv_rope: x row stride %lld (>= %lld, 16-byte rows), "
                     "16-byte aligned workspace", (long long)ld_x, (long long)k_dim);
  rc = device_ok("nf4_gemm_qkv_rope");
  if (rc != TB_OK) return rc;
  a.a_tiles = a.a_rows / kBM;  // one head a tile
  const Plan p = make_plan(tokens, a.a_tiles, a.red_blocks, sm_count(), true);
  if (workspace_bytes < (int64_t)p.splits * tokens * a.a_rows * 4)
    return set_error(TB_EINVAL, "nf4_gemm_qkv_rope: workspace of %lld bytes, %lld needed",
                     (long long)workspace_bytes, (long long)p.splits * tokens * a.a_rows * 4);
  a.part = workspace;
  cudaStream_t st = as_stream(stream);
  rc = run_gemm(kPart, a, p, x, ld_x, packed, st, "nf4_gemm_qkv_rope");
  if (rc != TB_OK) return rc;
  QkvArgs f;
  f.part = workspace;
  f.splits = p.splits;
  f.tokens = (int)tokens;
  f.a_rows = a.a_rows;
  f.bias = bias;
  f.lora_q = lora_q;
  f.lora_v = lora_v;
  f.cosv = cos;
  f.sinv = sin;
  f.pos_idx = pos_idx;
  f.seq = (int)seq;
  f.nh = n_heads;
  f.nkv = n_kv;
  f.q_out = q;
  f.k_out = k;
  f.v_out = v;
  const int64_t total = tokens * (n_heads + 2 * n_kv) * 64;
  int64_t blocks = (total + 255) / 256;
  const int cap = resident_blocks(qkv_rope_finish, 256);
  if (blocks > cap) blocks = cap;
  return launch("qkv_rope_finish", qkv_rope_finish, dim3((unsigned)blocks), dim3(256), 0, st, f);
}

extern "C" int tb_nf4_gemm_variant(int32_t variant) {
  if (variant < 0 || variant > 1)
    return set_error(TB_EINVAL, "nf4_gemm_variant: %d (0 automatic splits, 1 no split)", variant);
  g_variant = variant;
  return TB_OK;
}
