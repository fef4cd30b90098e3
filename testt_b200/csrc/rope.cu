// QKV pack: LoRA add + rotary embedding + scatter into the padded [batch, heads, seq, d] layout,
// forward and backward, for sm_100a.
//
// Reference: solution/rope.py:24-75 (rope_pack_fwd_kernel), :78-128 (rope_pack_bwd_kernel),
// :136-176 (RopePack). One CTA per token (backward) or per padded slot (forward with a slot map),
// one thread per (head row, 8-dim group): thread t owns dims d0..d0+7 of one half of head row
// t / (d/16) and the matching dims of the other half (the rotation pairs x[d] with x[d + d/2]).
// For Qwen2.5-1.5B (12 q + 2 k + 2 v heads, d = 128) that is 128 threads whose loads are all
// independent, so a slot costs one memory latency; all loads and stores are 16-byte vectors. With a slot
// map (slot_tok) the forward kernel covers every padded slot and writes the zero rows of padding
// itself, which removes the three zero-fills of the outputs the reference does before its launch
// (solution/rope.py:141-143).
//
// Token-major mode (tb_rope_tokens_fwd / _bwd, no counterpart in the reference): the same
// arithmetic with q, k, v laid out [rows, heads, d], the packed layout of variable-length
// attention, so no padded slot is written or read.
#include "common.cuh"

namespace tb {
namespace {

constexpr int kMaxThreads = 512;

struct RopeDims {
  int64_t rows, batch, seq;
  int nh, nkv, d, half;
};

template <bool kLoraFp32>
__device__ __forceinline__ void load8_lora(const void *p, int64_t idx, float (&f)[8]) {
  if (kLoraFp32) {
    load8f(static_cast<const float *>(p) + idx, f);
  } else {
    load8h(static_cast<const uint16_t *>(p) + idx, f);
  }
}

__device__ __forceinline__ void zero8(float (&f)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) f[k] = 0.f;
}

// Element offset of head row h (of `heads`) of token tok at slot (b, t): the padded
// [batch, heads, seq, d] layout, or token-major [rows, heads, d].
__device__ __forceinline__ int64_t head_row(bool tokens, int64_t tok, int64_t b, int64_t t,
                                            int heads, int h, int64_t seq, int D) {
  return tokens ? (tok * heads + h) * (int64_t)D : ((b * heads + h) * seq + t) * (int64_t)D;
}

// The token's q/k/v inputs of head row hr (qkv row, plus the LoRA row for q and v), in fp32.
template <bool kLoraFp32>
__device__ __forceinline__ void load_head_row(const uint16_t *qkv, const void *lq, const void *lv,
                                              const RopeDims &dm, int64_t tok, int hr, int d0,
                                              float (&x1)[8], float (&x2)[8]) {
  const int D = dm.d, H = dm.half;
  const uint16_t *row = qkv + tok * (int64_t)(dm.nh + 2 * dm.nkv) * D + (int64_t)hr * D;
  load8h(row + d0, x1);
  load8h(row + H + d0, x2);
  const void *l = nullptr;
  int64_t li = 0;
  if (hr < dm.nh) {
    l = lq;
    li = tok * ((int64_t)dm.nh * D) + (int64_t)hr * D;
  } else if (hr >= dm.nh + dm.nkv) {
    l = lv;
    li = tok * ((int64_t)dm.nkv * D) + (int64_t)(hr - dm.nh - dm.nkv) * D;
  }
  if (l != nullptr) {
    float a[8], c[8];
    load8_lora<kLoraFp32>(l, li + d0, a);
    load8_lora<kLoraFp32>(l, li + H + d0, c);
#pragma unroll
    for (int e = 0; e < 8; ++e) { x1[e] = x1[e] + a[e]; x2[e] = x2[e] + c[e]; }
  }
}

// Zero rows of the padding slots (slot_tok < 0) among slots [p0, p1): a warp per slot, the
// warp's slots p0 + warp + i * nwarps; lane i reads slot i's token, so memory is waited on once.
__device__ __forceinline__ void zero_padding(const int32_t *__restrict__ slot_tok, uint16_t *q,
                                             uint16_t *k, uint16_t *v, const RopeDims &dm,
                                             const FastDiv &seq_div, int64_t p0, int64_t p1) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int D = dm.d, total = dm.nh + 2 * dm.nkv, vpr = D / 8;  // 16-byte stores per head row
  float zero[8];
  zero8(zero);
  for (int64_t base = p0 + warp; base < p1; base += 32LL * nwarps) {
    const int64_t mine = base + (int64_t)lane * nwarps;
    const int32_t tok_l = mine < p1 ? __ldg(slot_tok + mine) : 0;
    for (int i = 0; i < 32; ++i) {
      const int64_t p = base + (int64_t)i * nwarps;
      if (p >= p1) break;
      if (__shfl_sync(0xffffffffu, tok_l, i) >= 0) continue;  // a token's slot: its CTA writes it
      uint32_t b32, t32;
      seq_div.divmod((uint32_t)p, b32, t32);
      const int64_t b = b32, t = t32;
      for (int j = lane; j < total * vpr; j += 32) {
        const int hr = j / vpr, c = (j - hr * vpr) * 8;
        uint16_t *dst;
        if (hr < dm.nh) dst = q + head_row(false, 0, b, t, dm.nh, hr, dm.seq, D);
        else if (hr < dm.nh + dm.nkv) dst = k + head_row(false, 0, b, t, dm.nkv, hr - dm.nh, dm.seq, D);
        else dst = v + head_row(false, 0, b, t, dm.nkv, hr - dm.nh - dm.nkv, dm.seq, D);
        store8h(dst + c, zero);
      }
    }
  }
}

// One CTA per token (blockIdx < rows). Its input rows do not depend on its position, so they
// are loaded before the position arrives; the rotary rows of the position come after (a 512 KB
// table, L2-resident after the first tokens). With a slot map every CTA also zeroes the padding
// slots of its own range of zero_chunk slots (the grid covers them when there are more ranges
// than tokens), so the padding costs no CTAs or waves of its own. kTokens: token-major outputs.
template <bool kLoraFp32, bool kTokens>
__global__ void __launch_bounds__(kMaxThreads)
    rope_fwd_vec(const uint16_t *__restrict__ qkv, const void *__restrict__ lq,
                 const void *__restrict__ lv, const float *__restrict__ cosv,
                 const float *__restrict__ sinv, const int64_t *__restrict__ pos_idx,
                 const int32_t *__restrict__ slot_tok, uint16_t *__restrict__ q,
                 uint16_t *__restrict__ k, uint16_t *__restrict__ v, RopeDims dm, FastDiv seq_div,
                 int64_t zero_chunk) {
  pdl_wait();
  pdl_release();
  const int64_t slots = dm.batch * dm.seq;
  const int D = dm.d, H = dm.half;
  const int total = dm.nh + 2 * dm.nkv;
  if (slot_tok != nullptr) {
    const int64_t p0 = (int64_t)blockIdx.x * zero_chunk;
    if (p0 < slots) zero_padding(slot_tok, q, k, v, dm, seq_div, p0,
                                 p0 + zero_chunk < slots ? p0 + zero_chunk : slots);
  }
  if ((int64_t)blockIdx.x >= dm.rows) return;
  const int lph = H / 8;                    // threads per head row
  const int rows_per_pass = blockDim.x / lph;
  if ((int)threadIdx.x >= rows_per_pass * lph) return;  // no __syncthreads below
  const int64_t tok = blockIdx.x;
  const int d0 = (threadIdx.x % lph) * 8;
  const int hr0 = threadIdx.x / lph;
  const int64_t pos = __ldg(pos_idx + tok);
  float x1[8], x2[8];
  if (hr0 < total) load_head_row<kLoraFp32>(qkv, lq, lv, dm, tok, hr0, d0, x1, x2);
  if (pos < 0 || pos >= slots) return;  // out-of-range position: nothing to write
  uint32_t b32, t32;
  seq_div.divmod((uint32_t)pos, b32, t32);
  const int64_t b = b32, t = t32;
  float c1[8], c2[8], s1[8], s2[8];
  load8f(cosv + t * D + d0, c1);
  load8f(cosv + t * D + H + d0, c2);
  load8f(sinv + t * D + d0, s1);
  load8f(sinv + t * D + H + d0, s2);
  for (int hr = hr0; hr < total; hr += rows_per_pass) {
    if (hr != hr0) load_head_row<kLoraFp32>(qkv, lq, lv, dm, tok, hr, d0, x1, x2);
    uint16_t *dst;
    if (hr < dm.nh) {
      dst = q + head_row(kTokens, tok, b, t, dm.nh, hr, dm.seq, D);
    } else if (hr < dm.nh + dm.nkv) {
      dst = k + head_row(kTokens, tok, b, t, dm.nkv, hr - dm.nh, dm.seq, D);
    } else {
      dst = v + head_row(kTokens, tok, b, t, dm.nkv, hr - dm.nh - dm.nkv, dm.seq, D);
      store8h(dst + d0, x1);  // v: LoRA-added, not rotated
      store8h(dst + H + d0, x2);
      continue;
    }
    float o1[8], o2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      o1[e] = x1[e] * c1[e] - x2[e] * s1[e];
      o2[e] = x2[e] * c2[e] + x1[e] * s2[e];
    }
    store8h(dst + d0, o1);
    store8h(dst + H + d0, o2);
  }
}

template <bool kTokens>
__global__ void __launch_bounds__(kMaxThreads)
    rope_bwd_vec(const uint16_t *__restrict__ dq, const uint16_t *__restrict__ dk,
                 const uint16_t *__restrict__ dv, const float *__restrict__ cosv,
                 const float *__restrict__ sinv, const int64_t *__restrict__ pos_idx,
                 uint16_t *__restrict__ dqkv, RopeDims dm, FastDiv seq_div) {
  pdl_wait();
  pdl_release();
  const int64_t tok = blockIdx.x;
  const int64_t slots = dm.batch * dm.seq;
  const int D = dm.d, H = dm.half;
  const int lph = H / 8, rows_per_pass = blockDim.x / lph, d0 = (threadIdx.x % lph) * 8;
  if ((int)threadIdx.x >= rows_per_pass * lph) return;  // no __syncthreads below
  const int total = dm.nh + 2 * dm.nkv;
  const int hr0 = threadIdx.x / lph;
  const int64_t pos = __ldg(pos_idx + tok);
  // token-major gradients do not depend on the position: the first head row's are loaded
  // while the position is in flight
  float g1[8], g2[8];
  bool have = false;
  if (kTokens && hr0 < total) {
    const uint16_t *src = hr0 < dm.nh ? (dq ? dq + head_row(true, tok, 0, 0, dm.nh, hr0, 0, D) : nullptr)
                          : hr0 < dm.nh + dm.nkv
                              ? (dk ? dk + head_row(true, tok, 0, 0, dm.nkv, hr0 - dm.nh, 0, D) : nullptr)
                              : (dv ? dv + head_row(true, tok, 0, 0, dm.nkv, hr0 - dm.nh - dm.nkv, 0, D)
                                    : nullptr);
    if (src != nullptr) {
      load8h(src + d0, g1);
      load8h(src + H + d0, g2);
      have = true;
    }
  }
  const bool inside = pos >= 0 && pos < slots;
  uint32_t b32 = 0, t32 = 0;
  if (inside) seq_div.divmod((uint32_t)pos, b32, t32);
  const int64_t b = b32, t = t32;
  float c1[8], c2[8], s1[8], s2[8];
  load8f(cosv + t * D + d0, c1);
  load8f(cosv + t * D + H + d0, c2);
  load8f(sinv + t * D + d0, s1);
  load8f(sinv + t * D + H + d0, s2);
  const int64_t W = (int64_t)total * D;
  uint16_t *row = dqkv + tok * W;
  for (int hr = hr0; hr < total; hr += rows_per_pass) {
    const uint16_t *src;
    bool rotate = true;
    if (hr < dm.nh) {
      src = dq ? dq + head_row(kTokens, tok, b, t, dm.nh, hr, dm.seq, D) : nullptr;
    } else if (hr < dm.nh + dm.nkv) {
      src = dk ? dk + head_row(kTokens, tok, b, t, dm.nkv, hr - dm.nh, dm.seq, D) : nullptr;
    } else {
      src = dv ? dv + head_row(kTokens, tok, b, t, dm.nkv, hr - dm.nh - dm.nkv, dm.seq, D)
               : nullptr;
      rotate = false;
    }
    float o1[8], o2[8];
    if (src != nullptr && inside) {
      if (!(kTokens && hr == hr0 && have)) {
        load8h(src + d0, g1);
        load8h(src + H + d0, g2);
      }
    } else {
      zero8(g1);
      zero8(g2);
    }
    if (rotate) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        o1[e] = g1[e] * c1[e] + g2[e] * s2[e];
        o2[e] = g2[e] * c2[e] - g1[e] * s1[e];
      }
      store8h(row + (int64_t)hr * D + d0, o1);
      store8h(row + (int64_t)hr * D + H + d0, o2);
    } else {
      store8h(row + (int64_t)hr * D + d0, g1);
      store8h(row + (int64_t)hr * D + H + d0, g2);
    }
  }
}

// Element-granular versions for head sizes whose half is not a multiple of 8 (or unaligned
// buffers): one thread per (unit, head row, j < d/2).
__device__ __forceinline__ float lora_at(const void *p, bool fp32, int64_t i) {
  return fp32 ? static_cast<const float *>(p)[i]
              : __half2float(__ushort_as_half(static_cast<const uint16_t *>(p)[i]));
}

__device__ __forceinline__ uint16_t h16(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float f16(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__global__ void rope_fwd_any(const uint16_t *qkv, const void *lq, const void *lv, bool lora_fp32,
                             const float *cosv, const float *sinv, const int64_t *pos_idx,
                             const int32_t *slot_tok, uint16_t *q, uint16_t *k, uint16_t *v,
                             RopeDims dm, bool tokens) {
  pdl_wait();
  pdl_release();
  const int total = dm.nh + 2 * dm.nkv;
  const int64_t slots = dm.batch * dm.seq;
  const int64_t units = slot_tok ? slots : dm.rows;
  const int64_t n = units * total * dm.half;
  const int D = dm.d, H = dm.half;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % H);
    const int hr = (int)((i / H) % total);
    const int64_t unit = i / ((int64_t)H * total);
    int64_t tok, pos;
    if (slot_tok) {
      pos = unit;
      tok = slot_tok[unit];
    } else {
      tok = unit;
      pos = pos_idx[unit];
      if (pos < 0 || pos >= slots) continue;
    }
    const int64_t b = pos / dm.seq, t = pos % dm.seq;
    uint16_t *dst;
    if (hr < dm.nh) dst = q + head_row(tokens, tok, b, t, dm.nh, hr, dm.seq, D);
    else if (hr < dm.nh + dm.nkv) dst = k + head_row(tokens, tok, b, t, dm.nkv, hr - dm.nh, dm.seq, D);
    else dst = v + head_row(tokens, tok, b, t, dm.nkv, hr - dm.nh - dm.nkv, dm.seq, D);
    if (tok < 0 || tok >= dm.rows) {
      dst[j] = 0;
      dst[j + H] = 0;
      continue;
    }
    const uint16_t *row = qkv + tok * (int64_t)total * D + (int64_t)hr * D;
    float x1 = f16(row[j]), x2 = f16(row[j + H]);
    if (hr < dm.nh && lq) {
      const int64_t li = tok * ((int64_t)dm.nh * D) + (int64_t)hr * D;
      x1 = x1 + lora_at(lq, lora_fp32, li + j);
      x2 = x2 + lora_at(lq, lora_fp32, li + j + H);
    }
    if (hr >= dm.nh + dm.nkv) {
      if (lv) {
        const int64_t li = tok * ((int64_t)dm.nkv * D) + (int64_t)(hr - dm.nh - dm.nkv) * D;
        x1 = x1 + lora_at(lv, lora_fp32, li + j);
        x2 = x2 + lora_at(lv, lora_fp32, li + j + H);
      }
      dst[j] = h16(x1);
      dst[j + H] = h16(x2);
      continue;
    }
    const float c1 = cosv[t * D + j], c2 = cosv[t * D + H + j];
    const float s1 = sinv[t * D + j], s2 = sinv[t * D + H + j];
    dst[j] = h16(x1 * c1 - x2 * s1);
    dst[j + H] = h16(x2 * c2 + x1 * s2);
  }
}

__global__ void rope_bwd_any(const uint16_t *dq, const uint16_t *dk, const uint16_t *dv,
                             const float *cosv, const float *sinv, const int64_t *pos_idx,
                             uint16_t *dqkv, RopeDims dm, bool tokens) {
  pdl_wait();
  pdl_release();
  const int total = dm.nh + 2 * dm.nkv;
  const int64_t slots = dm.batch * dm.seq;
  const int64_t n = dm.rows * total * dm.half;
  const int D = dm.d, H = dm.half;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % H);
    const int hr = (int)((i / H) % total);
    const int64_t tok = i / ((int64_t)H * total);
    const int64_t pos = pos_idx[tok];
    const bool inside = pos >= 0 && pos < slots;
    const int64_t b = inside ? pos / dm.seq : 0, t = inside ? pos % dm.seq : 0;
    const uint16_t *src;
    bool rotate = true;
    if (hr < dm.nh) src = dq ? dq + head_row(tokens, tok, b, t, dm.nh, hr, dm.seq, D) : nullptr;
    else if (hr < dm.nh + dm.nkv)
      src = dk ? dk + head_row(tokens, tok, b, t, dm.nkv, hr - dm.nh, dm.seq, D) : nullptr;
    else {
      src = dv ? dv + head_row(tokens, tok, b, t, dm.nkv, hr - dm.nh - dm.nkv, dm.seq, D)
               : nullptr;
      rotate = false;
    }
    const float g1 = (src && inside) ? f16(src[j]) : 0.f;
    const float g2 = (src && inside) ? f16(src[j + H]) : 0.f;
    uint16_t *row = dqkv + tok * (int64_t)total * D + (int64_t)hr * D;
    if (rotate) {
      const float c1 = cosv[t * D + j], c2 = cosv[t * D + H + j];
      const float s1 = sinv[t * D + j], s2 = sinv[t * D + H + j];
      row[j] = h16(g1 * c1 + g2 * s2);
      row[j + H] = h16(g2 * c2 - g1 * s1);
    } else {
      row[j] = h16(g1);
      row[j + H] = h16(g2);
    }
  }
}

__global__ void slot_scatter(const int64_t *pos_idx, int64_t rows, int64_t slots,
                             int32_t *slot_tok) {
  pdl_wait();
  pdl_release();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = pos_idx[i];
    if (p >= 0 && p < slots) slot_tok[p] = (int32_t)i;
  }
}

int check_dims(const char *what, int64_t rows, int64_t batch, int64_t seq, int nh, int nkv, int d) {
  if (rows < 0 || batch < 0 || seq <= 0 || nh <= 0 || nkv < 0 || d <= 0 || d % 2)
    return set_error(TB_EINVAL, "%s: bad dims rows=%lld batch=%lld seq=%lld nh=%d nkv=%d d=%d",
                     what, (long long)rows, (long long)batch, (long long)seq, nh, nkv, d);
  if (rows > 0x7fffffffLL || batch * seq > 0x7fffffffLL)
    return set_error(TB_EINVAL, "%s: too many rows or slots", what);
  return TB_OK;
}

// Threads of a per-unit CTA: one per (head row, 8-dim group), a warp multiple, at most
// kMaxThreads (more head rows loop).
int rope_threads(const RopeDims &dm) {
  int64_t t = (int64_t)(dm.nh + 2 * dm.nkv) * (dm.half / 8);
  t = ((t + 31) / 32) * 32;
  if (t > kMaxThreads) t = (kMaxThreads / (dm.half / 8)) * (dm.half / 8);
  return (int)t;
}

unsigned grid_for(int64_t n, int threads) {
  int64_t blocks = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 32;
  if (blocks > cap) blocks = cap;
  return (unsigned)(blocks > 0 ? blocks : 1);
}

}  // namespace
}  // namespace tb

using namespace tb;

namespace tb {
namespace {

int rope_fwd_launch(const char *what, bool tokens, const uint16_t *qkv, const void *lora_q,
                    const void *lora_v, int32_t lora_is_fp32, const float *cos, const float *sin,
                    const int64_t *pos_idx, const int32_t *slot_tok, uint16_t *q, uint16_t *k,
                    uint16_t *v, int64_t rows, int64_t batch, int64_t seq, int32_t n_heads,
                    int32_t n_kv, int32_t head_dim, void *stream) {
  int rc = check_dims(what, rows, batch, seq, n_heads, n_kv, head_dim);
  if (rc != TB_OK) return rc;
  if (!cos || !sin || !q || (n_kv > 0 && (!k || !v)))
    return set_error(TB_EINVAL, "%s: cos, sin, q, k, v are required", what);
  if (rows > 0 && (!qkv || !pos_idx))
    return set_error(TB_EINVAL, "%s: qkv and pos_idx are required", what);
  const int64_t units = slot_tok ? batch * seq : rows;
  if (units == 0) return TB_OK;
  RopeDims dm{rows, batch, seq, n_heads, n_kv, head_dim, head_dim / 2};
  const bool vec = dm.half % 8 == 0 && dm.half <= 8 * kMaxThreads && aligned(qkv, 16) && aligned(cos, 16) &&
                   aligned(sin, 16) && aligned(q, 16) && (n_kv == 0 || (aligned(k, 16) && aligned(v, 16))) &&
                   (!lora_q || aligned(lora_q, 16)) && (!lora_v || aligned(lora_v, 16));
  cudaStream_t st = as_stream(stream);
  if (vec) {
    // one CTA per token; with a slot map each CTA also zeroes the padding of an equal range of
    // slots (the grid grows past the tokens only when the ranges would exceed 32 slots a warp)
    const int threads = rope_threads(dm);
    int64_t ctas = rows, zero_chunk = 1;
    if (!tokens && slot_tok) {
      const int64_t slots = batch * seq, cap = 32LL * (threads / 32);
      zero_chunk = (slots + (rows > 0 ? rows : 1) - 1) / (rows > 0 ? rows : 1);
      if (zero_chunk > cap) zero_chunk = cap;
      const int64_t ranges = (slots + zero_chunk - 1) / zero_chunk;
      if (ranges > ctas) ctas = ranges;
    }
    const unsigned blocks = (unsigned)ctas;
    const FastDiv sd((uint32_t)seq);
    const int32_t *slots_map = tokens ? nullptr : slot_tok;
#define TB_ROPE_FWD(F, T)                                                                      \
  launch(what, rope_fwd_vec<F, T>, blocks, threads, 0, st, qkv, lora_q, lora_v, cos, sin,      \
         pos_idx, slots_map, q, k, v, dm, sd, zero_chunk)
    if (tokens) return lora_is_fp32 ? TB_ROPE_FWD(true, true) : TB_ROPE_FWD(false, true);
    return lora_is_fp32 ? TB_ROPE_FWD(true, false) : TB_ROPE_FWD(false, false);
#undef TB_ROPE_FWD
  }
  const int64_t n = units * (n_heads + 2 * n_kv) * (int64_t)dm.half;
  return launch(what, rope_fwd_any, grid_for(n, 256), 256, 0, st, qkv, lora_q, lora_v,
                lora_is_fp32 != 0, cos, sin, pos_idx, slot_tok, q, k, v, dm, tokens);
}

int rope_bwd_launch(const char *what, bool tokens, const uint16_t *dq, const uint16_t *dk,
                    const uint16_t *dv, const float *cos, const float *sin, const int64_t *pos_idx,
                    uint16_t *dqkv, int64_t rows, int64_t batch, int64_t seq, int32_t n_heads,
                    int32_t n_kv, int32_t head_dim, void *stream) {
  int rc = check_dims(what, rows, batch, seq, n_heads, n_kv, head_dim);
  if (rc != TB_OK) return rc;
  if (rows == 0) return TB_OK;
  if (!cos || !sin || !pos_idx || !dqkv)
    return set_error(TB_EINVAL, "%s: cos, sin, pos_idx, dqkv are required", what);
  RopeDims dm{rows, batch, seq, n_heads, n_kv, head_dim, head_dim / 2};
  const bool vec = dm.half % 8 == 0 && dm.half <= 8 * kMaxThreads && aligned(dqkv, 16) && aligned(cos, 16) &&
                   aligned(sin, 16) && (!dq || aligned(dq, 16)) && (!dk || aligned(dk, 16)) &&
                   (!dv || aligned(dv, 16));
  cudaStream_t st = as_stream(stream);
  if (vec) {
    const FastDiv sd((uint32_t)seq);
    if (tokens)
      return launch(what, rope_bwd_vec<true>, (unsigned)rows, rope_threads(dm), 0, st, dq, dk, dv,
                    cos, sin, pos_idx, dqkv, dm, sd);
    return launch(what, rope_bwd_vec<false>, (unsigned)rows, rope_threads(dm), 0, st, dq, dk, dv,
                  cos, sin, pos_idx, dqkv, dm, sd);
  }
  const int64_t n = rows * (n_heads + 2 * n_kv) * (int64_t)dm.half;
  return launch(what, rope_bwd_any, grid_for(n, 256), 256, 0, st, dq, dk, dv, cos, sin, pos_idx,
                dqkv, dm, tokens);
}

}  // namespace
}  // namespace tb

extern "C" int tb_rope_pack_fwd(const uint16_t *qkv, const void *lora_q, const void *lora_v,
                                int32_t lora_is_fp32, const float *cos, const float *sin,
                                const int64_t *pos_idx, const int32_t *slot_tok, uint16_t *q,
                                uint16_t *k, uint16_t *v, int64_t rows, int64_t batch, int64_t seq,
                                int32_t n_heads, int32_t n_kv, int32_t head_dim, void *stream) {
  return rope_fwd_launch("rope_pack_fwd", false, qkv, lora_q, lora_v, lora_is_fp32, cos, sin,
                         pos_idx, slot_tok, q, k, v, rows, batch, seq, n_heads, n_kv, head_dim,
                         stream);
}

extern "C" int tb_rope_pack_bwd(const uint16_t *dq, const uint16_t *dk, const uint16_t *dv,
                                const float *cos, const float *sin, const int64_t *pos_idx,
                                uint16_t *dqkv, int64_t rows, int64_t batch, int64_t seq,
                                int32_t n_heads, int32_t n_kv, int32_t head_dim, void *stream) {
  return rope_bwd_launch("rope_pack_bwd", false, dq, dk, dv, cos, sin, pos_idx, dqkv, rows, batch,
                         seq, n_heads, n_kv, head_dim, stream);
}

extern "C" int tb_rope_tokens_fwd(const uint16_t *qkv, const void *lora_q, const void *lora_v,
                                  int32_t lora_is_fp32, const float *cos, const float *sin,
                                  const int64_t *pos_idx, uint16_t *q, uint16_t *k, uint16_t *v,
                                  int64_t rows, int64_t batch, int64_t seq, int32_t n_heads,
                                  int32_t n_kv, int32_t head_dim, void *stream) {
  return rope_fwd_launch("rope_tokens_fwd", true, qkv, lora_q, lora_v, lora_is_fp32, cos, sin,
                         pos_idx, nullptr, q, k, v, rows, batch, seq, n_heads, n_kv, head_dim,
                         stream);
}

extern "C" int tb_rope_tokens_bwd(const uint16_t *dq, const uint16_t *dk, const uint16_t *dv,
                                  const float *cos, const float *sin, const int64_t *pos_idx,
                                  uint16_t *dqkv, int64_t rows, int64_t batch, int64_t seq,
                                  int32_t n_heads, int32_t n_kv, int32_t head_dim, void *stream) {
  return rope_bwd_launch("rope_tokens_bwd", true, dq, dk, dv, cos, sin, pos_idx, dqkv, rows,
                         batch, seq, n_heads, n_kv, head_dim, stream);
}

extern "C" int tb_slot_index(const int64_t *pos_idx, int64_t rows, int64_t slots,
                             int32_t *slot_tok, void *stream) {
  if (rows < 0 || slots < 0) return set_error(TB_EINVAL, "slot_index: negative size");
  if (slots == 0) return TB_OK;
  if (!slot_tok || (rows > 0 && !pos_idx))
    return set_error(TB_EINVAL, "slot_index: pos_idx and slot_tok are required");
  cudaStream_t st = as_stream(stream);
  if (cudaMemsetAsync(slot_tok, 0xff, (size_t)slots * sizeof(int32_t), st) != cudaSuccess)
    return check_launch("slot_index memset");
  if (rows == 0) return TB_OK;
  return launch("slot_index", slot_scatter, grid_for(rows, 256), 256, 0, st, pos_idx, rows, slots,
                slot_tok);
}
