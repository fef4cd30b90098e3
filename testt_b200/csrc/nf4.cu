// NF4 unpack (bitsandbytes 4-bit layout, plain or nested absmax) for sm_100a.
//
// Reference: solution/nf4.py:27-45 (nf4_unpack_kernel) and :72-105 (unpack_into /
// unpack_concat). The reference runs one Triton program per 1024 packed bytes and one launch per
// weight; here one launch covers every weight of a stacked GEMM operand (q|k|v, gate|up).
//
// Layout of the work: a warp handles a span of 32 * kUnroll consecutive 4-byte words of one
// weight; lane l takes words l, l + 32, l + 64, ... of the span, so every 4-byte load and every
// 16-byte store of a warp instruction is contiguous (128 B in, 512 B out). Contiguous stores
// matter most here (80 % of the bytes are the fp16 output): giving each thread 16 contiguous
// packed bytes instead made every store instruction 64-byte strided and cost 1.5x on B200.
// Each weight's range of words is padded to whole spans, so the weight of a span is uniform
// across the warp and found once per span; the 256-entry nested code table, the offset and the
// 16-entry NF4 table live in shared memory, block indices use 32-bit invariant division
// (FastDiv). Sizes or alignments that do not fit take a byte-granular kernel.
// Arithmetic is bit-exact with the reference: each mul/add rounded on its own (__fmul_rn /
// __fadd_rn, no FMA contraction), then one round-to-nearest-even to fp16.
#include "common.cuh"

namespace tb {
namespace {

#ifndef TB_NF4_UNROLL
#define TB_NF4_UNROLL 8
#endif

constexpr int kMaxW = TB_NF4_MAX_WEIGHTS;
constexpr int kUnroll = TB_NF4_UNROLL;  // words per lane per warp span (4 or 8)
constexpr int kThreads = 256;
static_assert(kUnroll == 4 || kUnroll == 8, "a span's blocks of 64 must fit one lane each");

struct Nf4Job {
  int n;
  const uint8_t *packed[kMaxW];
  const float *absmax_f32[kMaxW];
  const uint8_t *absmax_u8[kMaxW];
  const float *code2[kMaxW];
  const float *absmax2[kMaxW];
  const float *offset[kMaxW];
  const float *table[kMaxW];
  uint16_t *out[kMaxW];
  int64_t start[kMaxW + 1];  // prefix sums of units (padded words for the word kernel, else bytes)
  uint32_t n_words[kMaxW];   // words of each weight (word kernel)
  FastDiv block_div[kMaxW];  // packed byte index -> absmax block (divisor qblock / 2)
  FastDiv nest_div[kMaxW];   // absmax block -> nested block (divisor qblock2)
};

__device__ __forceinline__ int find_weight(const Nf4Job &job, int64_t u) {
  int j = 0;
#pragma unroll
  for (int i = 1; i < kMaxW; ++i)
    if (i < job.n && u >= job.start[i]) j = i;
  return j;
}

__device__ __forceinline__ float block_scale(const Nf4Job &job, int j, uint32_t b) {
  if (job.absmax_f32[j] != nullptr) return __ldg(job.absmax_f32[j] + b);
  const int code = __ldg(job.absmax_u8[j] + b);
  const float a = __fmul_rn(__ldg(job.code2[j] + code), __ldg(job.absmax2[j] + job.nest_div[j].div(b)));
  return __fadd_rn(a, __ldg(job.offset[j]));
}

constexpr int kSpan = 32 * kUnroll;  // words per warp span

// Shared-memory address tab | byte b of x: byte b of x moved to byte 0 and bytes 1..3 taken from
// tab (256-byte aligned, so its byte 0 is zero), one byte permute.
__device__ __forceinline__ uint32_t table_addr(uint32_t x, uint32_t tab, int b) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(tab), "r"(0x7650u | (uint32_t)b));
  return r;
}

// fp16 values of the 8 nibbles of `word` (high nibble of each byte first) times `scale`, packed.
// `tab` is the shared-memory address of the 16-entry table (256-byte aligned). The byte offsets
// 4 * nibble of all eight nibbles come from two shift-and-mask operations (each byte of lo4 /
// hi4 holds one), and each lookup address from one byte permute.
__device__ __forceinline__ uint4 decode_word(uint32_t word, float scale, uint32_t tab) {
  const uint32_t lo4 = (word << 2) & 0x3c3c3c3cu;
  const uint32_t hi4 = (word >> 2) & 0x3c3c3c3cu;
  float f[8];
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    float hi, lo;
    asm("ld.shared.f32 %0, [%1];" : "=f"(hi) : "r"(table_addr(hi4, tab, b)));
    asm("ld.shared.f32 %0, [%1];" : "=f"(lo) : "r"(table_addr(lo4, tab, b)));
    // two products per instruction (sm_100 packed fp32 multiply, each lane rounded to nearest
    // even exactly like __fmul_rn)
    const float2 p = __fmul2_rn(make_float2(hi, lo), make_float2(scale, scale));
    f[2 * b] = p.x;
    f[2 * b + 1] = p.y;
  }
  return make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]), pack_half2(f[4], f[5]),
                    pack_half2(f[6], f[7]));
}

#ifndef TB_NF4_SPANS
#define TB_NF4_SPANS 2
#endif
constexpr int kSpansPerWarp = TB_NF4_SPANS;  // spans a warp is sized to take (grid sizing)
#ifndef TB_NF4_WAVES
#define TB_NF4_WAVES 1
#endif
constexpr int kWavesCap = TB_NF4_WAVES;  // grid at most this many waves of resident blocks

// One warp span of blocksize-64 weights, loaded ahead of its decode: the span's words and the
// absmax of lane l's block (block first/8 + l): the fp32 absmax (plain) or the u8 code and the
// fp32 absmax2 it scales (nested).
struct Span64 {
  int j;
  uint32_t first, nwords;
  uint32_t word[kUnroll];
  float a;
  int code;  // -1: plain absmax (or no block for this lane)
};

__device__ __forceinline__ void fetch_span64(const Nf4Job &job, int64_t sp, int lane, Span64 &s) {
  s.j = find_weight(job, sp * kSpan);  // uniform across the warp
  s.first = (uint32_t)(sp * kSpan - job.start[s.j]);
  s.nwords = job.n_words[s.j];
  const uint32_t *src = reinterpret_cast<const uint32_t *>(job.packed[s.j]);
#pragma unroll
  for (int k = 0; k < kUnroll; ++k) {
    const uint32_t local = s.first + k * 32 + lane;
    s.word[k] = local < s.nwords ? __ldg(src + local) : 0u;
  }
  const uint32_t b = (s.first >> 3) + lane;
  s.a = 0.f;
  s.code = -1;
  if (lane < 4 * kUnroll && b * 8 < s.nwords) {
    if (job.absmax_f32[s.j] != nullptr) {
      s.a = __ldg(job.absmax_f32[s.j] + b);
    } else {
      s.code = __ldg(job.absmax_u8[s.j] + b);
      s.a = __ldg(job.absmax2[s.j] + job.nest_div[s.j].div(b));
    }
  }
}

// Blocksize 64 with the next span's loads issued before the current span's decode, so a warp
// keeps its memory latency behind its own arithmetic. A span of 32 * kUnroll words holds
// 4 * kUnroll blocks: lane l computes the scale of block l once and word k of lane l (block
// 4k + l/8) takes it by shuffle.
__global__ void __launch_bounds__(kThreads) nf4_unpack_words64(const __grid_constant__ Nf4Job job) {
  pdl_wait();
  pdl_release();
  __shared__ __align__(256) float table[kMaxW][64];  // 16 entries used, 256-byte stride
  __shared__ float code2[kMaxW][256];
  __shared__ float offs[kMaxW];
  for (int i = threadIdx.x; i < job.n * 16; i += blockDim.x)
    table[i >> 4][i & 15] = __ldg(job.table[i >> 4] + (i & 15));
  for (int j = 0; j < job.n; ++j) {
    if (job.absmax_f32[j] != nullptr) continue;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) code2[j][i] = __ldg(job.code2[j] + i);
    if (threadIdx.x == 0) offs[j] = __ldg(job.offset[j]);
  }
  __syncthreads();

  const int64_t spans = job.start[job.n] / kSpan;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (kThreads / 32);
  const uint32_t table_base = (uint32_t)__cvta_generic_to_shared(&table[0][0]);
  int64_t sp = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  if (sp >= spans) return;
  Span64 cur, nxt;
  fetch_span64(job, sp, lane, cur);
  while (true) {
    const int64_t nsp = sp + warps;
    const bool more = nsp < spans;  // uniform across the warp
    if (more) fetch_span64(job, nsp, lane, nxt);
    float mine = cur.a;
    if (cur.code >= 0) mine = __fadd_rn(__fmul_rn(code2[cur.j][cur.code], cur.a), offs[cur.j]);
    const uint32_t tab = table_base + (uint32_t)cur.j * 256u;
    uint4 *dst = reinterpret_cast<uint4 *>(job.out[cur.j]);
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const float scale = __shfl_sync(0xffffffffu, mine, 4 * k + (lane >> 3));
      const uint32_t local = cur.first + k * 32 + lane;
      // plain stores, not streaming ones: the GEMMs that follow read these weights, and part of
      // them can still be in L2 (captured step 8.476 / 8.478 ms with evict-first stores against
      // 8.463 / 8.465 ms, same box)
      if (local < cur.nwords) dst[local] = decode_word(cur.word[k], scale, tab);
    }
    if (!more) break;
    cur = nxt;
    sp = nsp;
  }
}

// Any even blocksize: each word's absmax block is found by invariant division and its scale
// computed by the lane itself.
__global__ void __launch_bounds__(kThreads) nf4_unpack_words_any(const __grid_constant__ Nf4Job job) {
  pdl_wait();
  pdl_release();
  __shared__ __align__(256) float table[kMaxW][64];  // 16 entries used, 256-byte stride
  __shared__ float code2[kMaxW][256];
  __shared__ float offs[kMaxW];
  for (int i = threadIdx.x; i < job.n * 16; i += blockDim.x)
    table[i >> 4][i & 15] = __ldg(job.table[i >> 4] + (i & 15));
  for (int j = 0; j < job.n; ++j) {
    if (job.absmax_f32[j] != nullptr) continue;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) code2[j][i] = __ldg(job.code2[j] + i);
    if (threadIdx.x == 0) offs[j] = __ldg(job.offset[j]);
  }
  __syncthreads();

  const int64_t spans = job.start[job.n] / kSpan;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (kThreads / 32);
  for (int64_t sp = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); sp < spans;
       sp += warps) {
    const int j = find_weight(job, sp * kSpan);  // uniform across the warp
    const uint32_t first = (uint32_t)(sp * kSpan - job.start[j]);
    const uint32_t nwords = job.n_words[j];
    const uint32_t *src = reinterpret_cast<const uint32_t *>(job.packed[j]);
    const bool plain = job.absmax_f32[j] != nullptr;
    const uint32_t tab = (uint32_t)__cvta_generic_to_shared(&table[j][0]);
    uint4 *dst = reinterpret_cast<uint4 *>(job.out[j]);
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const uint32_t local = first + k * 32 + lane;
      if (local >= nwords) continue;
      const uint32_t word = __ldg(src + local);
      const uint32_t b = job.block_div[j].div(local * 4u);
      float scale;
      if (plain) {
        scale = __ldg(job.absmax_f32[j] + b);
      } else {
        const int code = __ldg(job.absmax_u8[j] + b);
        const float a2 = __ldg(job.absmax2[j] + job.nest_div[j].div(b));
        scale = __fadd_rn(__fmul_rn(code2[j][code], a2), offs[j]);
      }
      dst[local] = decode_word(word, scale, tab);
    }
  }
}

// Byte-granular path for sizes or alignments the word kernel cannot take.
__global__ void __launch_bounds__(kThreads) nf4_unpack_bytes(const __grid_constant__ Nf4Job job) {
  pdl_wait();
  pdl_release();
  const int64_t total = job.start[job.n];
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total; u += stride) {
    const int j = find_weight(job, u);
    const uint32_t local = (uint32_t)(u - job.start[j]);
    const float scale = block_scale(job, j, job.block_div[j].div(local));
    const uint32_t byte = __ldg(job.packed[j] + local);
    const float hi = __fmul_rn(__ldg(job.table[j] + (byte >> 4)), scale);
    const float lo = __fmul_rn(__ldg(job.table[j] + (byte & 15u)), scale);
    job.out[j][2 * (size_t)local] = __half_as_ushort(__float2half_rn(hi));
    job.out[j][2 * (size_t)local + 1] = __half_as_ushort(__float2half_rn(lo));
  }
}

int launch_job(Nf4Job &job, const int64_t *n_bytes, const int32_t *half_qblock, cudaStream_t stream) {
  bool words = true;
  for (int j = 0; j < job.n; ++j) {
    words = words && n_bytes[j] % 4 == 0 && half_qblock[j] % 4 == 0 &&
            aligned(job.packed[j], 4) && aligned(job.out[j], 16);
  }
  job.start[0] = 0;
  for (int j = 0; j < job.n; ++j) {
    int64_t units = n_bytes[j];
    if (words) {
      job.n_words[j] = (uint32_t)(n_bytes[j] / 4);
      units = ((n_bytes[j] / 4 + kSpan - 1) / kSpan) * kSpan;  // whole warp spans
    }
    job.start[j + 1] = job.start[j] + units;
  }
  for (int j = job.n; j < kMaxW; ++j) job.start[j + 1] = job.start[job.n];
  const int64_t total = job.start[job.n];
  if (total == 0) return TB_OK;
  // one block per 8 spans (words) or 256 bytes of work, at most what is resident at once,
  // then a grid-stride loop
  bool block64 = true;
  for (int j = 0; j < job.n; ++j) block64 = block64 && half_qblock[j] == 32;
  const int64_t per_block = (int64_t)kThreads * (words ? kUnroll : 1);
  int64_t blocks = (total + per_block - 1) / per_block;
  if (words && block64) {
    // about kSpansPerWarp spans per warp, but at least one block per SM
    static int cap = resident_blocks(nf4_unpack_words64, kThreads) * kWavesCap;
    const int64_t per = (int64_t)(kThreads / 32) * kSpansPerWarp;
    blocks = (total / kSpan + per - 1) / per;
    if (blocks < sm_count()) blocks = sm_count();
    if (blocks > cap) blocks = cap;
    return launch("nf4_unpack", nf4_unpack_words64, (unsigned)blocks, kThreads, 0, stream, job);
  }
  if (words) {
    static int cap = resident_blocks(nf4_unpack_words_any, kThreads);
    if (blocks > cap) blocks = cap;
    return launch("nf4_unpack", nf4_unpack_words_any, (unsigned)blocks, kThreads, 0, stream, job);
  }
  static int cap = resident_blocks(nf4_unpack_bytes, kThreads);
  if (blocks > cap) blocks = cap;
  return launch("nf4_unpack", nf4_unpack_bytes, (unsigned)blocks, kThreads, 0, stream, job);
}

int fill_common(Nf4Job &job, int j, const uint8_t *packed, const float *table, uint16_t *out,
                int64_t n_bytes, int32_t qblock) {
  if (qblock <= 0 || qblock % 2)
    return set_error(TB_EINVAL, "nf4_unpack: weight %d: blocksize %d must be positive and even", j,
                     qblock);
  if (n_bytes < 0 || n_bytes >= (1LL << 32))
    return set_error(TB_EINVAL, "nf4_unpack: weight %d: n_bytes %lld out of range [0, 2^32)", j,
                     (long long)n_bytes);
  if (packed == nullptr || table == nullptr || out == nullptr)
    return set_error(TB_EINVAL, "nf4_unpack: weight %d: packed, nf4 table and out are required", j);
  job.packed[j] = packed;
  job.table[j] = table;
  job.out[j] = out;
  job.block_div[j] = FastDiv((uint32_t)(qblock / 2));
  job.absmax_f32[j] = nullptr;
  job.absmax_u8[j] = nullptr;
  job.code2[j] = nullptr;
  job.absmax2[j] = nullptr;
  job.offset[j] = nullptr;
  job.nest_div[j] = FastDiv(1);
  return TB_OK;
}

int fill_nested(Nf4Job &job, int j, const uint8_t *absmax_u8, const float *code2,
                const float *absmax2, const float *offset, int32_t qblock2) {
  if (qblock2 <= 0)
    return set_error(TB_EINVAL, "nf4_unpack: weight %d: nested blocksize %d", j, qblock2);
  if (absmax_u8 == nullptr || code2 == nullptr || absmax2 == nullptr || offset == nullptr)
    return set_error(TB_EINVAL,
                     "nf4_unpack: weight %d: nested layout needs absmax_u8, code2, absmax2, offset",
                     j);
  job.absmax_u8[j] = absmax_u8;
  job.code2[j] = code2;
  job.absmax2[j] = absmax2;
  job.offset[j] = offset;
  job.nest_div[j] = FastDiv((uint32_t)qblock2);
  return TB_OK;
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" int tb_nf4_unpack_nested(const uint8_t *packed, const uint8_t *absmax_u8,
                                    const float *code2, const float *absmax2, const float *offset,
                                    const float *nf4_table, uint16_t *out, int64_t n_bytes,
                                    int32_t qblock, int32_t qblock2, void *stream) {
  Nf4Job job{};
  job.n = 1;
  int rc = fill_common(job, 0, packed, nf4_table, out, n_bytes, qblock);
  if (rc == TB_OK) rc = fill_nested(job, 0, absmax_u8, code2, absmax2, offset, qblock2);
  if (rc != TB_OK) return rc;
  const int32_t half = qblock / 2;
  return launch_job(job, &n_bytes, &half, as_stream(stream));
}

extern "C" int tb_nf4_unpack_plain(const uint8_t *packed, const float *absmax,
                                   const float *nf4_table, uint16_t *out, int64_t n_bytes,
                                   int32_t qblock, void *stream) {
  Nf4Job job{};
  job.n = 1;
  int rc = fill_common(job, 0, packed, nf4_table, out, n_bytes, qblock);
  if (rc != TB_OK) return rc;
  if (absmax == nullptr) return set_error(TB_EINVAL, "nf4_unpack_plain: absmax is required");
  job.absmax_f32[0] = absmax;
  const int32_t half = qblock / 2;
  return launch_job(job, &n_bytes, &half, as_stream(stream));
}

extern "C" int tb_nf4_unpack_multi(int32_t n_weights, const uint8_t *const *packed,
                                   const float *const *absmax_f32,
                                   const uint8_t *const *absmax_u8, const float *const *code2,
                                   const float *const *absmax2, const float *const *offset,
                                   const float *const *nf4_table, uint16_t *const *out,
                                   const int64_t *n_bytes, const int32_t *qblock,
                                   const int32_t *qblock2, void *stream) {
  if (n_weights < 1 || n_weights > kMaxW)
    return set_error(TB_EINVAL, "nf4_unpack_multi: %d weights (1..%d allowed)", n_weights, kMaxW);
  if (packed == nullptr || nf4_table == nullptr || out == nullptr || n_bytes == nullptr ||
      qblock == nullptr)
    return set_error(TB_EINVAL, "nf4_unpack_multi: packed, nf4_table, out, n_bytes, qblock required");
  Nf4Job job{};
  job.n = n_weights;
  int32_t half[kMaxW];
  for (int j = 0; j < n_weights; ++j) {
    int rc = fill_common(job, j, packed[j], nf4_table[j], out[j], n_bytes[j], qblock[j]);
    if (rc != TB_OK) return rc;
    half[j] = qblock[j] / 2;
    const float *plain = absmax_f32 ? absmax_f32[j] : nullptr;
    if (plain != nullptr) {
      job.absmax_f32[j] = plain;
    } else {
      if (!absmax_u8 || !code2 || !absmax2 || !offset || !qblock2)
        return set_error(TB_EINVAL, "nf4_unpack_multi: weight %d has neither layout", j);
      rc = fill_nested(job, j, absmax_u8[j], code2[j], absmax2[j], offset[j], qblock2[j]);
      if (rc != TB_OK) return rc;
    }
  }
  return launch_job(job, n_bytes, half, as_stream(stream));
}
