// NF4-weight GEMMs on the 5th-generation tensor cores with the NF4 decode in the operand
// producer, so the fp16 copy of a frozen weight is never written to HBM:
//
//   forward   out[t, n] = fp16(sum_k x[t, k] W[n, k] (+ bias[n]))   FrozenNF4Linear.forward,
//                                                                 solution/nf4.py:115-118
//   backward  out[t, k] = fp16(sum_n dy[t, n] W[n, k])              FrozenNF4Linear.backward,
//                                                                 solution/nf4.py:121-127
//
// W is up to four NF4 weights stacked by rows (q|k|v, gate|up), each in bitsandbytes' packing
// (row-major, blocksize 64, element 2i in the high nibble of byte i) with fp32 absmax per block.
// A nested state's absmax is expanded once by the caller (code2[c] * absmax2[b / 256] + offset,
// each operation rounded on its own, as the unpack kernel does), so every decoded value is
// fp16(table[q] * absmax) rounded once: bit-identical to tb_nf4_unpack_*'s output, and the
// product differs from cuBLAS over the unpacked weight only by the order of the fp32 sums.
//
// The MMA computes D[a, t] = A[a, :] . B[t, :]. A is a 128-row tile of the decoded weight
// (output features forward, input features backward) and B the token operand (x or dy), both
// K-major with the 128-byte swizzle. The skinny token dimension is the MMA's N, so each decoded
// weight tile serves up to 384 tokens (two N <= 192 sub-tiles, or one N <= 256).
//
// CTA = (128 A rows, a group of <= 384 tokens, one split of the reduction); 6 warps:
//   warp 0      TMA producer of the token tiles (nsub sub-tiles of BN rows x 64) per stage
//   warp 1      TMEM allocation (512 columns), MMA issue (M128 N=BN K16), commits
//   warps 2..5  decoders: NF4 words and absmax read from global memory two stages ahead,
//               decoded to fp16 and stored into the stage's A tile in the swizzled layout the
//               MMA descriptor reads (fence.proxy.async, then an arrive on the stage's A
//               barrier); afterwards the epilogue: TMEM -> fp16 output (one split).
// A split reduction (small projections: the grid is filled by splitting the reduction) sums
// its splits' accumulators either within a thread-block cluster of the splits (the default):
// each CTA parks its fp32 accumulator in its now idle stage buffers, and CTA r of the cluster
// adds column slice r of all of them through distributed shared memory in split order, with
// the bias; or through fp32 partials [split, token, row] in a caller's workspace, summed in
// split order by nf4_gemm_reduce (tb_nf4_gemm_variant(1)).
// tb_nf4_gemm_qkv_rope runs the q|k|v projection with its bias, the LoRA rows and the rotary
// embedding in the finishing phase (one head a tile), writing token-major q, k, v.
// tb_nf4_gemm_swiglu runs the MLP's GEMMs with SwiGLU in the epilogue: the gate|up forward
// (tiles of 64 gate and 64 up rows, act formed from both halves through shared memory) and
// down's dX (dact never written: the epilogue applies the in-place SwiGLU backward to gu).
// Every mbarrier wait is bounded (mbar_wait); a role that gives up sets the CTA's error flag
// and leaves its loop, every role meets at the final barrier and TMEM is always released.
// No multicast is used.
#include <cuda.h>

#include <cstddef>

#include "common.cuh"

namespace tb {
namespace {

constexpr int kMaxW = 4;
constexpr int kBM = 128;                        // A rows per CTA
constexpr int kBK = 64;                         // reduction per stage: 128 bytes of fp16
constexpr int kStages = 3;
constexpr int kMaxSpan = 384;                   // tokens per CTA
constexpr int kABytes = kBM * kBK * 2;          // 16 KB
constexpr int kBBytes = kMaxSpan * kBK * 2;     // 48 KB
constexpr int kThreads = 192;
constexpr int kDecoders = 128;                  // warps 2..5
constexpr int kTmemCols = 512;

struct Smem {
  alignas(1024) uint8_t a[kStages][kABytes];
  alignas(1024) uint8_t b[kStages][kBBytes];
  alignas(256) float table[kMaxW][64];          // 16 entries used; 256-byte aligned rows
  uint64_t full_a[kStages], full_b[kStages], empty[kStages];
  uint64_t acc_full, mma_done;
  uint32_t tmem_base;
  volatile int error;
};
// the cluster reduction keeps a CTA's fp32 accumulator [span][128] in the stage buffers a, b
static_assert(offsetof(Smem, b) == sizeof(Smem::a), "stage buffers a and b are contiguous");
static_assert(sizeof(Smem::a) + sizeof(Smem::b) >= (size_t)kMaxSpan * kBM * 4,
              "the stage buffers hold a whole accumulator");

struct GemmArgs {
  const uint8_t *packed[kMaxW];
  const float *absmax[kMaxW];
  const float *table[kMaxW];
  int row_start[kMaxW + 1];  // first stacked W row of each weight; row_start[n_w] = all rows
  int n_w;
  int k_dim;                 // columns of W
  int a_rows;                // rows of the A operand: row_start[n_w] forward, k_dim backward
  int red_blocks;            // reduction blocks of 64
  int tokens;
  int bn, nsub, span, splits;
  uint32_t idesc;
  const uint16_t *bias;      // forward with one split only (else nf4_gemm_reduce adds it)
  uint16_t *out;
  int64_t ld_out;
  float *part;               // [splits, tokens, a_rows] fp32 when splits > 1 (not cluster)
  int cluster;               // splits > 1: the splits are one thread-block cluster and sum
                             // their accumulators through distributed shared memory
  int mode;                  // kPlain, kSwigluFwd, kSwigluBwd (one split), kQkvRope
  uint16_t *gu;              // SwiGLU modes: fp16 [tokens, 2 * inter] gate | up (row stride ld_gu)
  int64_t ld_gu;
  int inter;
  // kQkvRope: W = (q, k, v) with heads of 128 rows, one head a tile; the finished values (plus
  // bias) are rounded to fp16 as the GEMM's output, the LoRA rows added (q, v) and q, k rotated,
  // then written token-major: q [tokens, nh, 128], k, v [tokens, nkv, 128]
  const uint16_t *lora_q, *lora_v;  // fp16 [tokens, nh * 128], [tokens, nkv * 128] or NULL
  const float *cosv, *sinv;         // [seq, 128]
  const int64_t *pos_idx;           // [tokens]: padded position, t = pos % seq
  int seq, nh, nkv;
  uint16_t *q_out, *k_out, *v_out;
};

// kSwigluFwd: W = (gate, up); CTA x holds gate rows 64x .. 64x + 63 as A rows 0-63 and the same
//   up rows as A rows 64-127; the epilogue writes gu = fp16(x [gate|up]^T) and
//   act = fp16(silu(g) u) to out (mlp.py:31-40 on the GEMM's fp16 output).
// kSwigluBwd: W = (down,), transposed: the epilogue rounds dact = dy . W_down to fp16 and applies
//   the in-place SwiGLU backward to gu (mlp.py:43-58).
constexpr int kPlain = 0, kSwigluFwd = 1, kSwigluBwd = 2, kQkvRope = 3;

// ---- tcgen05 / TMA helpers (PTX ISA: tcgen05.mma, cp.async.bulk.tensor) --------------------

// K-major, 128-byte-swizzle operand descriptor: start address, LBO 1 (unused for swizzled
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

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// every thread of every CTA of the cluster; orders shared-memory writes before the barrier
// with the reads (local or remote) after it. The non-.aligned form: the lanes of the producer
// and MMA warps reach it at different times.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// the float at the address `p` has in this CTA, in the shared memory of cluster CTA `rank`
__device__ __forceinline__ float ld_cluster(const float *p, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(p)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
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

// barrier of the four epilogue warps (named barrier 1, 128 threads)
__device__ __forceinline__ void epilogue_sync() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ int weight_of(const GemmArgs &args, int row) {
  int j = 0;
#pragma unroll
  for (int i = 1; i < kMaxW; ++i)
    if (i < args.n_w && row >= args.row_start[i]) j = i;
  return j;
}

// Forward: decoder thread d owns A row d (one output feature) of the tile: per stage the 32
// packed bytes of its row's 64 columns and their one absmax.
struct FwdRaw {
  uint4 lo, hi;
  float scale;
};

__device__ __forceinline__ void load_fwd(const GemmArgs &args, const uint8_t *row_bytes,
                                         const float *row_absmax, int blk, FwdRaw &r) {
  const uint4 *p = reinterpret_cast<const uint4 *>(row_bytes + (size_t)blk * 32);
  r.lo = __ldg(p);
  r.hi = __ldg(p + 1);
  r.scale = __ldg(row_absmax + blk);
}

// Row d of the tile, 8 words -> 8 swizzled 16-byte chunks (chunk c of row d at c ^ (d % 8)).
__device__ __forceinline__ void decode_fwd(const FwdRaw &r, uint32_t a_tile, int d, uint32_t tab) {
  const uint32_t w[8] = {r.lo.x, r.lo.y, r.lo.z, r.lo.w, r.hi.x, r.hi.y, r.hi.z, r.hi.w};
  const uint32_t base = a_tile + (uint32_t)(d >> 3) * 1024u + (uint32_t)(d & 7) * 128u;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    st_shared16(base + ((uint32_t)(c ^ (d & 7)) << 4), decode_word(w[c], r.scale, tab));
}

// Backward: the stage's reduction block is 64 W rows (n) and the tile 128 W columns (k).
// Decoder thread d = 8 * k8 + n8 takes the 8 x 8 block of rows n8*8.. and columns k8*8..: one
// 4-byte word of each of its 8 rows, decoded and transposed in registers into 8 chunks (one per
// column k, holding that column's 8 rows), stored to A rows k8*8.. at chunk n8. Lanes with
// consecutive n8 store to 8 different 16-byte positions: conflict-free 16-byte stores.
struct BwdRaw {
  uint32_t w[8];
  float s[8];
  int j;
};

__device__ __forceinline__ void load_bwd(const GemmArgs &args, int blk, int a0, int n8, int k8,
                                         BwdRaw &r) {
  const int n_first = blk * kBK;  // stacked W row
  r.j = weight_of(args, n_first);
  const int local = n_first - args.row_start[r.j] + n8 * 8;
  const size_t row_bytes = (size_t)(args.k_dim >> 1);
  const int kblocks = args.k_dim >> 6;
  const uint8_t *src = args.packed[r.j] + (size_t)local * row_bytes + (size_t)((a0 >> 1) + 4 * k8);
  const float *am = args.absmax[r.j] + (size_t)local * kblocks + (a0 >> 6) + (k8 >> 3);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    r.w[i] = __ldg(reinterpret_cast<const uint32_t *>(src + (size_t)i * row_bytes));
    r.s[i] = __ldg(am + (size_t)i * kblocks);
  }
}

__device__ __forceinline__ void decode_bwd(const BwdRaw &r, uint32_t a_tile, int n8, int k8,
                                           uint32_t tab) {
  uint32_t h[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint4 v = decode_word(r.w[i], r.s[i], tab);  // row n8*8+i, columns k8*8 .. +7
    h[i][0] = v.x;
    h[i][1] = v.y;
    h[i][2] = v.z;
    h[i][3] = v.w;
  }
  const uint32_t base = a_tile + (uint32_t)k8 * 1024u;
#pragma unroll
  for (int q = 0; q < 4; ++q) {  // columns 2q, 2q + 1
    uint32_t even[4], odd[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {  // rows 2p, 2p + 1
      even[p] = prmt(h[2 * p][q], h[2 * p + 1][q], 0x5410u);  // (row 2p, row 2p+1) of column 2q
      odd[p] = prmt(h[2 * p][q], h[2 * p + 1][q], 0x7632u);   // ... of column 2q + 1
    }
    const int k0 = 2 * q, k1 = 2 * q + 1;
    st_shared16(base + (uint32_t)k0 * 128u + ((uint32_t)(n8 ^ k0) << 4),
                make_uint4(even[0], even[1], even[2], even[3]));
    st_shared16(base + (uint32_t)k1 * 128u + ((uint32_t)(n8 ^ k1) << 4),
                make_uint4(odd[0], odd[1], odd[2], odd[3]));
  }
}

template <bool kTrans>
__global__ void __launch_bounds__(kThreads, 1)
    nf4_gemm_kernel(const __grid_constant__ CUtensorMap map_b, const __grid_constant__ GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                        ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int a0 = blockIdx.x * kBM;
  const int t0 = blockIdx.y * args.span;
  const int split = blockIdx.z;
  const int q = args.red_blocks / args.splits, rem = args.red_blocks % args.splits;
  const int first = split * q + (split < rem ? split : rem);
  const int nblk = q + (split < rem ? 1 : 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full_a[s], kDecoders);
      mbar_init(&sm.full_b[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.acc_full, 1);
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
    // ---- TMA producer of the token tiles ------------------------------------------------
    if (lane == 0) {
      const uint32_t bytes = (uint32_t)(args.nsub * args.bn * kBK * 2);
      int issued = 0;
      for (int i = 0; i < nblk && !sm.error; ++i) {
        const int s = i % kStages;
        const uint32_t parity = (uint32_t)((i / kStages) & 1);
        if (!mbar_wait(&sm.empty[s], parity ^ 1)) {
          sm.error = 1;
          break;
        }
        mbar_expect_tx(&sm.full_b[s], bytes);
        for (int j = 0; j < args.nsub; ++j)
          tma_load_2d(smem_u32(sm.b[s]) + (uint32_t)(j * args.bn * kBK * 2), &map_b,
                      (first + i) * kBK, t0 + j * args.bn, &sm.full_b[s]);
        ++issued;
      }
      // every copy issued must have landed before the CTA may leave (bounded)
      for (int i = issued - (issued < kStages ? issued : kStages); i < issued; ++i)
        mbar_wait(&sm.full_b[i % kStages], (uint32_t)((i / kStages) & 1));
    }
  } else if (warp == 1) {
    // ---- MMA issuer -----------------------------------------------------------------------
    if (lane == 0) {
      for (int i = 0; i < nblk && !sm.error; ++i) {
        const int s = i % kStages;
        const uint32_t parity = (uint32_t)((i / kStages) & 1);
        if (!mbar_wait(&sm.full_b[s], parity) || !mbar_wait(&sm.full_a[s], parity)) {
          sm.error = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a_tile = smem_u32(sm.a[s]);
        const uint32_t b_tile = smem_u32(sm.b[s]);
        for (int j = 0; j < args.nsub; ++j) {
          const uint32_t d = tmem + (uint32_t)(j * args.bn);
          const uint32_t bj = b_tile + (uint32_t)(j * args.bn * kBK * 2);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)  // K = 16 per MMA: 32 bytes along the swizzled row
            mma_f16(d, smem_desc(a_tile + k * 32), smem_desc(bj + k * 32), args.idesc,
                    (i | k) != 0);
        }
        mma_commit(&sm.empty[s]);  // A and B of the stage are free once these MMAs have read them
      }
      mma_commit(&sm.acc_full);
      mma_commit(&sm.mma_done);
      // no MMA in flight before TMEM is released; a wait that gives up is recorded (the MMAs
      // depend on nothing that could stall them, so this only guards against the impossible)
      if (!mbar_wait(&sm.mma_done, 0)) sm.error = 1;
    }
  } else {
    // ---- decoders, then the epilogue --------------------------------------------------------
    const int d = threadIdx.x - 64;  // 0 .. 127
    if (!kTrans) {
      // a tile lies inside one weight (rows % 128 == 0), or holds 64 gate and 64 up rows
      const bool inter = args.mode == kSwigluFwd;
      const int j = inter ? (d < 64 ? 0 : 1) : weight_of(args, a0);
      const int local = inter ? (int)blockIdx.x * 64 + (d & 63) : a0 - args.row_start[j] + d;
      const uint8_t *row_bytes = args.packed[j] + (size_t)local * (size_t)(args.k_dim >> 1);
      const float *row_absmax = args.absmax[j] + (size_t)local * (size_t)(args.k_dim >> 6);
      const uint32_t tab = smem_u32(&sm.table[j][0]);
      FwdRaw r0{}, r1{};
      if (nblk > 0) load_fwd(args, row_bytes, row_absmax, first, r0);
      if (nblk > 1) load_fwd(args, row_bytes, row_absmax, first + 1, r1);
      for (int i = 0; i < nblk && !sm.error; ++i) {
        FwdRaw r2{};
        if (i + 2 < nblk) load_fwd(args, row_bytes, row_absmax, first + i + 2, r2);
        const int s = i % kStages;
        if (!mbar_wait(&sm.empty[s], (uint32_t)(((i / kStages) & 1) ^ 1))) {
          sm.error = 1;
          break;
        }
        decode_fwd(r0, smem_u32(sm.a[s]), d, tab);
        fence_proxy_async();  // the generic-proxy stores, visible to the tensor core
        mbar_arrive(&sm.full_a[s]);
        r0 = r1;
        r1 = r2;
      }
    } else {
      const int n8 = d & 7, k8 = d >> 3;
      BwdRaw r0{}, r1{};
      if (nblk > 0) load_bwd(args, first, a0, n8, k8, r0);
      if (nblk > 1) load_bwd(args, first + 1, a0, n8, k8, r1);
      for (int i = 0; i < nblk && !sm.error; ++i) {
        BwdRaw r2{};
        if (i + 2 < nblk) load_bwd(args, first + i + 2, a0, n8, k8, r2);
        const int s = i % kStages;
        if (!mbar_wait(&sm.empty[s], (uint32_t)(((i / kStages) & 1) ^ 1))) {
          sm.error = 1;
          break;
        }
        decode_bwd(r0, smem_u32(sm.a[s]), n8, k8, smem_u32(&sm.table[r0.j][0]));
        fence_proxy_async();
        mbar_arrive(&sm.full_a[s]);
        r0 = r1;
        r1 = r2;
      }
    }

    // epilogue: warp w reads TMEM lanes 32 * (w % 4) .. (its quarter of the A rows)
    const int quarter = warp & 3;
    const int ok = mbar_wait(&sm.acc_full, 0) ? 1 : 0;
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) sm.error = 1;
    }
    const bool go = __all_sync(0xffffffffu, ok) && !sm.error;
    if (args.mode == kSwigluFwd) {
      // phase 1: every warp stores its fp16 values to gu; the up warps (quarters 2, 3) also to
      // xch[column][64] in the idle stage buffers. Phase 2 (after the epilogue warps' barrier,
      // reached by all four whatever happened): the gate warps form act.
      uint16_t *xch = reinterpret_cast<uint16_t *>(&sm.a[0][0]);
      const bool up = quarter >= 2;
      const int fl = (quarter & 1) * 32 + lane;     // feature within the tile's 64
      const int f = (int)blockIdx.x * 64 + fl;
      if (go) {
        tc_fence_after();
        for (int j = 0; j < args.nsub; ++j)
          for (int c = 0; c < args.bn; c += 32) {
            const int tb = t0 + j * args.bn + c;
            if (tb >= args.tokens) break;
            uint32_t v[32];
            tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(j * args.bn + c), v);
            const int ne = args.tokens - tb < 32 ? args.tokens - tb : 32;
            uint16_t *o = args.gu + (int64_t)tb * args.ld_gu + (up ? args.inter : 0) + f;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              if (e >= ne) break;
              const uint16_t x16 = f2h(__uint_as_float(v[e]));
              o[(int64_t)e * args.ld_gu] = x16;
              if (up) xch[(j * args.bn + c + e) * 64 + fl] = x16;
            }
          }
      }
      epilogue_sync();
      if (go && !up) {
        for (int j = 0; j < args.nsub; ++j)
          for (int c = 0; c < args.bn; c += 32) {
            const int tb = t0 + j * args.bn + c;
            if (tb >= args.tokens) break;
            uint32_t v[32];
            tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(j * args.bn + c), v);
            const int ne = args.tokens - tb < 32 ? args.tokens - tb : 32;
            uint16_t *o = args.out + (int64_t)tb * args.ld_out + f;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              if (e >= ne) break;
              const float g = h2f(f2h(__uint_as_float(v[e])));
              const float u = h2f(xch[(j * args.bn + c + e) * 64 + fl]);
              o[(int64_t)e * args.ld_out] = f2h(silu(g) * u);
            }
          }
      }
    } else if (args.mode == kSwigluBwd) {
      // dact rounded to fp16 as the unfused GEMM's output; gu's two halves updated in place,
      // 16 tokens at a time with all their loads issued before the math
      if (go) {
        tc_fence_after();
        const int f = a0 + quarter * 32 + lane;
        for (int j = 0; j < args.nsub; ++j)
          for (int c = 0; c < args.bn; c += 32) {
            const int tb = t0 + j * args.bn + c;
            if (tb >= args.tokens) break;
            uint32_t v[32];
            tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(j * args.bn + c), v);
            const int ne = args.tokens - tb < 32 ? args.tokens - tb : 32;
            uint16_t *pg = args.gu + (int64_t)tb * args.ld_gu + f;
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
    } else if (go) {
      tc_fence_after();
      const int row = a0 + quarter * 32 + lane;
      const bool add_bias = args.splits == 1 && args.bias != nullptr;
      const float bias = add_bias ? __half2float(__ushort_as_half(__ldg(args.bias + row))) : 0.f;
      for (int j = 0; j < args.nsub; ++j) {
        for (int c = 0; c < args.bn; c += 32) {
          const int tb = t0 + j * args.bn + c;
          if (tb >= args.tokens) break;  // uniform across the warp
          uint32_t v[32];
          tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(j * args.bn + c), v);
          const int ne = args.tokens - tb < 32 ? args.tokens - tb : 32;
          if (args.cluster || args.mode == kQkvRope) {
            // the stage buffers are free once every MMA has completed: the accumulator goes
            // to red[column][row] (a warp's lanes are consecutive rows: conflict-free)
            float *red = reinterpret_cast<float *>(&sm.a[0][0]);
            const int col0 = j * args.bn + c;
#pragma unroll
            for (int e = 0; e < 32; ++e) red[(col0 + e) * kBM + quarter * 32 + lane] = __uint_as_float(v[e]);
          } else if (args.splits == 1) {
            uint16_t *o = args.out + (int64_t)tb * args.ld_out + row;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              if (e >= ne) break;
              float x = __uint_as_float(v[e]);
              if (add_bias) x = __fadd_rn(x, bias);
              o[(int64_t)e * args.ld_out] = __half_as_ushort(__float2half_rn(x));
            }
          } else {
            float *p = args.part + ((int64_t)split * args.tokens + tb) * args.a_rows + row;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              if (e >= ne) break;
              p[(int64_t)e * args.a_rows] = __uint_as_float(v[e]);
            }
          }
        }
      }
    }
  }

  if (args.mode == kQkvRope) {
    // one head per tile: CTA r of the cluster (or the CTA alone) finishes columns
    // [r * per, (r + 1) * per): rows p and p + 64 of a token together (the rotation's pair)
    if (args.cluster) cluster_sync(); else __syncthreads();
    const int parts = args.cluster ? args.splits : 1;
    const int per = (args.span + parts - 1) / parts;
    const int c_lo = (args.cluster ? (int)cluster_ctarank() : 0) * per;
    const int c_hi = c_lo + per < args.span ? c_lo + per : args.span;
    const float *red = reinterpret_cast<const float *>(&sm.a[0][0]);
    const int hr = blockIdx.x;
    const int D = kBM, H = kBM / 2;
    for (int e = threadIdx.x; e < (c_hi - c_lo) * H; e += kThreads) {
      const int col = c_lo + e / H, pr = e % H;
      const int tok = t0 + col;
      if (tok >= args.tokens) break;  // columns ascend with e
      float s1 = 0.f, s2 = 0.f;
      for (int q = 0; q < parts; ++q) {
        const float *base = red + col * kBM;
        s1 = __fadd_rn(s1, args.cluster ? ld_cluster(base + pr, (uint32_t)q) : base[pr]);
        s2 = __fadd_rn(s2, args.cluster ? ld_cluster(base + pr + H, (uint32_t)q) : base[pr + H]);
      }
      if (args.bias != nullptr) {
        s1 = __fadd_rn(s1, h2f(__ldg(args.bias + hr * D + pr)));
        s2 = __fadd_rn(s2, h2f(__ldg(args.bias + hr * D + pr + H)));
      }
      float x1 = h2f(f2h(s1)), x2 = h2f(f2h(s2));  // the GEMM's fp16 output
      const uint16_t *lora = nullptr;
      uint16_t *dst;
      if (hr < args.nh) {
        lora = args.lora_q ? args.lora_q + ((int64_t)tok * args.nh + hr) * D : nullptr;
        dst = args.q_out + ((int64_t)tok * args.nh + hr) * D;
      } else if (hr < args.nh + args.nkv) {
        dst = args.k_out + ((int64_t)tok * args.nkv + hr - args.nh) * D;
      } else {
        const int hv = hr - args.nh - args.nkv;
        lora = args.lora_v ? args.lora_v + ((int64_t)tok * args.nkv + hv) * D : nullptr;
        dst = args.v_out + ((int64_t)tok * args.nkv + hv) * D;
      }
      if (lora != nullptr) {
        x1 = x1 + h2f(__ldg(lora + pr));
        x2 = x2 + h2f(__ldg(lora + pr + H));
      }
      float o1 = x1, o2 = x2;  // v: LoRA-added, not rotated
      if (hr < args.nh + args.nkv) {
        const int64_t pos = __ldg(args.pos_idx + tok);
        if (pos < 0) continue;  // no position: nothing written (as tb_rope_tokens_fwd)
        const int64_t t = pos % args.seq;
        const float c1 = __ldg(args.cosv + t * D + pr), c2 = __ldg(args.cosv + t * D + H + pr);
        const float n1 = __ldg(args.sinv + t * D + pr), n2 = __ldg(args.sinv + t * D + H + pr);
        o1 = x1 * c1 - x2 * n1;
        o2 = x2 * c2 + x1 * n2;
      }
      dst[pr] = f2h(o1);
      dst[pr + H] = f2h(o2);
    }
    if (args.cluster) cluster_sync();
  } else if (args.cluster) {
    // the splits' sums: cluster CTA r finishes columns [r * per, (r + 1) * per) of the tile,
    // adding the CTAs' accumulators in rank (= split) order, then the bias; the second barrier
    // keeps every CTA's shared memory alive until all have read it
    cluster_sync();
    const int per = (args.span + args.splits - 1) / args.splits;
    const int c_lo = (int)cluster_ctarank() * per;
    const int c_hi = c_lo + per < args.span ? c_lo + per : args.span;
    const float *red = reinterpret_cast<const float *>(&sm.a[0][0]);
    for (int e = threadIdx.x; e < (c_hi - c_lo) * kBM; e += kThreads) {
      const int col = c_lo + e / kBM, r = e % kBM;
      const int t = t0 + col;
      if (t >= args.tokens) break;  // columns ascend with e
      float sum = 0.f;
      for (int q = 0; q < args.splits; ++q)
        sum = __fadd_rn(sum, ld_cluster(red + col * kBM + r, (uint32_t)q));
      if (args.bias != nullptr)
        sum = __fadd_rn(sum, __half2float(__ushort_as_half(__ldg(args.bias + a0 + r))));
      args.out[(int64_t)t * args.ld_out + a0 + r] = __half_as_ushort(__float2half_rn(sum));
    }
    cluster_sync();
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

// fp16 row-major [rows, cols] with row stride ld (elements) -> box [box_rows, 64], 128-byte
// swizzle; rows past the end read as zeros.
int make_map(CUtensorMap *map, const void *base, int64_t rows, int64_t cols, int64_t ld,
             int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return set_error(TB_EDEVICE, "nf4_gemm: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                        strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TB_EINVAL, "nf4_gemm: tensor map encode failed (%d)", (int)r);
  return TB_OK;
}

struct Plan {
  int bn, nsub, span, groups, splits, cluster;
};

// 0: automatic (split partials summed within a cluster), 1: split partials through the
// workspace and nf4_gemm_reduce, 2: cluster always (process-wide; tb_nf4_gemm_variant)
int g_variant = 0;
constexpr int kMaxCluster = 8;  // portable cluster size

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Tokens in groups of <= 384 (one or two sub-tiles of a multiple of 32 tokens); the reduction
// split until the grid reaches one CTA per SM (at least 4 blocks of 64 a split), within the
// workspace.
Plan make_plan(int64_t tokens, int a_tiles, int red_blocks, int64_t a_rows, int64_t ws_bytes,
               int sms, int variant) {
  Plan p;
  p.groups = (int)ceil_div(tokens, kMaxSpan);
  const int64_t tg = ceil_div(tokens, p.groups);
  if (tg <= 256) {
    p.nsub = 1;
    p.bn = (int)ceil_div(tg, 32) * 32;
  } else {
    p.nsub = 2;
    p.bn = (int)ceil_div(ceil_div(tg, 2), 32) * 32;
  }
  p.span = p.nsub * p.bn;
  const int64_t base = (int64_t)a_tiles * p.groups;
  int splits = 1;
  if (base < sms) {
    splits = (int)(sms / base);
    const int most = red_blocks / 4 > 1 ? red_blocks / 4 : 1;
    if (splits > most) splits = most;
    if (splits > 16) splits = 16;
  }
  const bool cluster = variant != 1;
  if (cluster) {
    if (splits > kMaxCluster) splits = kMaxCluster;
  } else {
    while (splits > 1 && (int64_t)splits * tokens * a_rows * 4 > ws_bytes) --splits;
  }
  p.splits = splits;
  p.cluster = cluster && splits > 1;
  return p;
}

}  // namespace

TB_REGISTER_TIMEOUT_READER(nf4_gemm)

}  // namespace tb

using namespace tb;

namespace {

// Shared argument checks; fills the weight table of `a`. Returns TB_OK or an error.
int gemm_args(int32_t transpose, int64_t tokens, int32_t n_weights, const uint8_t *const *packed,
              const float *const *absmax, const float *const *nf4_table, const int64_t *rows,
              int64_t k_dim, GemmArgs &a) {
  if (n_weights < 1 || n_weights > kMaxW || !packed || !absmax || !nf4_table || !rows)
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
    if (!packed[j] || !absmax[j] || !nf4_table[j])
      return set_error(TB_EINVAL, "nf4_gemm: weight %d has a missing pointer", j);
    if (rows[j] <= 0 || rows[j] % r_align != 0)
      return set_error(TB_EINVAL, "nf4_gemm: weight %d has %lld rows (a multiple of %lld needed)",
                       j, (long long)rows[j], (long long)r_align);
    if (!aligned(packed[j], transpose ? 4 : 16) || !aligned(absmax[j], 4) ||
        !aligned(nf4_table[j], 4))
      return set_error(TB_EALIGN, "nf4_gemm: weight %d is not aligned", j);
    a.packed[j] = packed[j];
    a.absmax[j] = absmax[j];
    a.table[j] = nf4_table[j];
    total += rows[j];
    if (total > (1LL << 24)) return set_error(TB_EINVAL, "nf4_gemm: too many rows");
    a.row_start[j + 1] = (int)total;
  }
  for (int j = n_weights; j < kMaxW; ++j) {
    a.packed[j] = nullptr;
    a.absmax[j] = nullptr;
    a.table[j] = nullptr;
    a.row_start[j + 1] = (int)total;
  }
  a.n_w = n_weights;
  a.k_dim = (int)k_dim;
  a.a_rows = transpose ? (int)k_dim : (int)total;
  a.red_blocks = transpose ? (int)(total / kBK) : (int)(k_dim / kBK);
  a.tokens = (int)tokens;
  return TB_OK;
}

}  // namespace

extern "C" int64_t tb_nf4_gemm_workspace(int32_t transpose, int64_t tokens, int32_t n_weights,
                                         const int64_t *rows, int64_t k_dim) {
  if (n_weights < 1 || n_weights > kMaxW || rows == nullptr || tokens <= 0 || k_dim <= 0) return 0;
  int64_t total = 0;
  for (int j = 0; j < n_weights; ++j) total += rows[j];
  const int64_t a_rows = transpose ? k_dim : total;
  const int red_blocks = (int)((transpose ? total : k_dim) / kBK);
  const Plan p = make_plan(tokens, (int)(a_rows / kBM), red_blocks, a_rows, INT64_MAX, sm_count(),
                           g_variant);
  return p.splits > 1 && !p.cluster ? (int64_t)p.splits * tokens * a_rows * 4 : 0;
}

extern "C" int tb_nf4_gemm(int32_t transpose, const uint16_t *tokens_in, int64_t tokens,
                           int64_t ld_in, int32_t n_weights, const uint8_t *const *packed,
                           const float *const *absmax, const float *const *nf4_table,
                           const int64_t *rows, int64_t k_dim, const uint16_t *bias, uint16_t *out,
                           int64_t ld_out, float *workspace, int64_t workspace_bytes,
                           void *stream) {
  GemmArgs a;
  int rc = gemm_args(transpose, tokens, n_weights, packed, absmax, nf4_table, rows, k_dim, a);
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
  int dev = 0, major = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return set_error(TB_EDEVICE, "nf4_gemm: needs an sm_100 GPU");

  const int a_tiles = a.a_rows / kBM;
  const Plan p = make_plan(tokens, a_tiles, a.red_blocks, a.a_rows,
                           workspace ? workspace_bytes : 0, sm_count(), g_variant);
  a.bn = p.bn;
  a.nsub = p.nsub;
  a.span = p.span;
  a.splits = p.splits;
  a.idesc = (1u << 4) | ((uint32_t)(p.bn >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
  a.bias = bias;
  a.out = out;
  a.ld_out = ld_out;
  a.part = p.splits > 1 && !p.cluster ? workspace : nullptr;
  a.cluster = p.cluster;
  a.mode = kPlain;
  a.gu = nullptr;
  a.ld_gu = 0;
  a.inter = 0;
  a.lora_q = a.lora_v = nullptr;
  a.cosv = a.sinv = nullptr;
  a.pos_idx = nullptr;
  a.seq = a.nh = a.nkv = 0;
  a.q_out = a.k_out = a.v_out = nullptr;

  CUtensorMap map_b;
  rc = make_map(&map_b, tokens_in, tokens, red_dim, ld_in, p.bn);
  if (rc != TB_OK) return rc;
  const size_t smem = sizeof(Smem) + 1024;
  auto kernel = transpose ? nf4_gemm_kernel<true> : nf4_gemm_kernel<false>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return check_launch("nf4_gemm attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a_tiles, (unsigned)p.groups, (unsigned)p.splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;  // the splits of one (tile, token group) form a cluster
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)p.splits;
  cfg.attrs = attr;
  cfg.numAttrs = p.cluster ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, map_b, a);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return set_error(TB_ELAUNCH, "nf4_gemm: launch failed: %s", cudaGetErrorString(e));
  }
  if (p.splits == 1 || p.cluster) return TB_OK;
  const int64_t vecs = tokens * (a.a_rows / 8);
  const int64_t blocks64 = (vecs + 255) / 256;
  const int cap = resident_blocks(nf4_gemm_reduce, 256);
  const int blocks = (int)(blocks64 < cap ? blocks64 : cap);
  return launch("nf4_gemm_reduce", nf4_gemm_reduce, dim3((unsigned)blocks), dim3(256), 0,
                as_stream(stream), (const float *)workspace, p.splits, tokens, a.a_rows, bias, out,
                ld_out);
}

// The MLP's two NF4 GEMMs with SwiGLU in their epilogue (one split each):
//   forward  (backward == 0): weights (gate, up), each [inter, k_dim]; tokens_in = x
//            [tokens, k_dim]; writes gu = fp16(x [gate|up]^T) [tokens, 2 inter] (row stride
//            ld_gu) and act = fp16(silu(g) u) [tokens, inter] (row stride ld_act)
//   backward (backward == 1): weight (down,) [hidden, inter] (k_dim = inter); tokens_in = dy
//            [tokens, hidden]; dact = fp16(dy . W_down) stays in the epilogue, which overwrites
//            gu with d(gate|up) (act unused)
extern "C" int tb_nf4_gemm_swiglu(int32_t backward, const uint16_t *tokens_in, int64_t tokens,
                                  int64_t ld_in, int32_t n_weights, const uint8_t *const *packed,
                                  const float *const *absmax, const float *const *nf4_table,
                                  const int64_t *rows, int64_t k_dim, uint16_t *gu, int64_t ld_gu,
                                  uint16_t *act, int64_t ld_act, void *stream) {
  GemmArgs a;
  int rc = gemm_args(backward ? 1 : 0, tokens, n_weights, packed, absmax, nf4_table, rows, k_dim,
                     a);
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
  int dev = 0, major = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return set_error(TB_EDEVICE, "nf4_gemm_swiglu: needs an sm_100 GPU");

  // forward tiles hold 64 features of each weight; backward tiles 128 features of dact
  const int a_tiles = backward ? (int)(inter / kBM) : (int)(inter / 64);
  Plan p = make_plan(tokens, a_tiles, a.red_blocks, a.a_rows, 0, sm_count(), 1);
  p.splits = 1;
  p.cluster = 0;
  a.bn = p.bn;
  a.nsub = p.nsub;
  a.span = p.span;
  a.splits = 1;
  a.idesc = (1u << 4) | ((uint32_t)(p.bn >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
  a.bias = nullptr;
  a.out = act;
  a.ld_out = ld_act;
  a.part = nullptr;
  a.cluster = 0;
  a.mode = backward ? kSwigluBwd : kSwigluFwd;
  a.gu = gu;
  a.ld_gu = ld_gu;
  a.inter = (int)inter;
  a.lora_q = a.lora_v = nullptr;
  a.cosv = a.sinv = nullptr;
  a.pos_idx = nullptr;
  a.seq = a.nh = a.nkv = 0;
  a.q_out = a.k_out = a.v_out = nullptr;

  CUtensorMap map_b;
  rc = make_map(&map_b, tokens_in, tokens, red_dim, ld_in, p.bn);
  if (rc != TB_OK) return rc;
  const size_t smem = sizeof(Smem) + 1024;
  auto kernel = backward ? nf4_gemm_kernel<true> : nf4_gemm_kernel<false>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return check_launch("nf4_gemm_swiglu attribute");
  const dim3 grid((unsigned)a_tiles, (unsigned)p.groups, 1u);
  kernel<<<grid, kThreads, smem, as_stream(stream)>>>(map_b, a);
  return check_launch("nf4_gemm_swiglu");
}

// The q|k|v projection with its bias, the LoRA rows and the rotary embedding in the epilogue:
// weights (q, k, v) = [n_heads * 128, k_dim], [n_kv * 128, k_dim] twice; x [tokens, k_dim] (row
// stride ld_x); out q [tokens, n_heads, 128], k, v [tokens, n_kv, 128] (token-major, contiguous)
// = what tb_rope_tokens_fwd writes from the GEMM's fp16 output (solution/rope.py:24-75 with the
// padded scatter replaced by token-major rows). lora_q / lora_v fp16 or NULL; cos, sin fp32
// [seq, 128]; pos_idx int64 padded positions (t = pos % seq).
extern "C" int tb_nf4_gemm_qkv_rope(const uint16_t *x, int64_t tokens, int64_t ld_x,
                                    const uint8_t *const *packed, const float *const *absmax,
                                    const float *const *nf4_table, int64_t k_dim,
                                    const uint16_t *bias, const uint16_t *lora_q,
                                    const uint16_t *lora_v, const float *cos, const float *sin,
                                    const int64_t *pos_idx, int64_t seq, int32_t n_heads,
                                    int32_t n_kv, uint16_t *q, uint16_t *k, uint16_t *v,
                                    void *stream) {
  if (n_heads <= 0 || n_kv <= 0 || n_heads % n_kv != 0 || seq <= 0)
    return set_error(TB_EINVAL, "nf4_gemm_qkv_rope: heads %d kv %d seq %lld", n_heads, n_kv,
                     (long long)seq);
  const int64_t rows[3] = {(int64_t)n_heads * kBM, (int64_t)n_kv * kBM, (int64_t)n_kv * kBM};
  GemmArgs a;
  int rc = gemm_args(0, tokens, 3, packed, absmax, nf4_table, rows, k_dim, a);
  if (rc != TB_OK) return rc;
  if (tokens == 0) return TB_OK;
  if (!x || !cos || !sin || !pos_idx || !q || !k || !v)
    return set_error(TB_EINVAL, "nf4_gemm_qkv_rope: x, cos, sin, pos_idx, q, k, v required");
  if (ld_x < k_dim || ld_x % 8 != 0 || !aligned(x, 16))
    return set_error(TB_EINVAL, "nf4_gemm_qkv_rope: x row stride %lld (>= %lld, 16-byte rows)",
                     (long long)ld_x, (long long)k_dim);
  int dev = 0, major = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return set_error(TB_EDEVICE, "nf4_gemm_qkv_rope: needs an sm_100 GPU");

  const int a_tiles = a.a_rows / kBM;  // one head a tile
  const Plan p = make_plan(tokens, a_tiles, a.red_blocks, a.a_rows, 0, sm_count(), 0);
  a.bn = p.bn;
  a.nsub = p.nsub;
  a.span = p.span;
  a.splits = p.splits;
  a.cluster = p.cluster;
  a.idesc = (1u << 4) | ((uint32_t)(p.bn >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
  a.bias = bias;
  a.out = nullptr;
  a.ld_out = 0;
  a.part = nullptr;
  a.mode = kQkvRope;
  a.gu = nullptr;
  a.ld_gu = 0;
  a.inter = 0;
  a.lora_q = lora_q;
  a.lora_v = lora_v;
  a.cosv = cos;
  a.sinv = sin;
  a.pos_idx = pos_idx;
  a.seq = (int)seq;
  a.nh = n_heads;
  a.nkv = n_kv;
  a.q_out = q;
  a.k_out = k;
  a.v_out = v;

  CUtensorMap map_b;
  rc = make_map(&map_b, x, tokens, k_dim, ld_x, p.bn);
  if (rc != TB_OK) return rc;
  const size_t smem = sizeof(Smem) + 1024;
  if (cudaFuncSetAttribute(nf4_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return check_launch("nf4_gemm_qkv_rope attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a_tiles, (unsigned)p.groups, (unsigned)p.splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)p.splits;
  cfg.attrs = attr;
  cfg.numAttrs = p.cluster ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, nf4_gemm_kernel<false>, map_b, a);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return set_error(TB_ELAUNCH, "nf4_gemm_qkv_rope: launch failed: %s", cudaGetErrorString(e));
  }
  return TB_OK;
}

extern "C" int tb_nf4_gemm_variant(int32_t variant) {
  if (variant < 0 || variant > 2)
    return set_error(TB_EINVAL, "nf4_gemm_variant: %d (0 auto, 1 workspace, 2 cluster)", variant);
  g_variant = variant;
  return TB_OK;
}
