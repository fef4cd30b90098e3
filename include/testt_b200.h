/*
 * testt_b200 — C ABI of the B200 (sm_100a) kernels of the fused QLoRA hot path.
 *
 * Every entry point takes raw device pointers, 64-bit sizes, scalar parameters and a CUDA stream
 * (passed as `void *`, a `cudaStream_t`; NULL means the legacy default stream). Nothing is
 * allocated inside: the caller owns every buffer. Work is only enqueued; the call returns once
 * the launch is queued. The return value is TB_OK (0) or a negative TB_E* code; the text of the
 * last error on the calling host thread is returned by tb_last_error().
 *
 * fp16 tensors are passed as `uint16_t *` (IEEE binary16 bit patterns), so this header needs no
 * CUDA include. Reference citations (file:line) are into the SalReII/testt repository.
 */
#ifndef TESTT_B200_H
#define TESTT_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TB_OK 0
#define TB_EINVAL (-1)   /* bad size, shape or missing required pointer            */
#define TB_EALIGN (-2)   /* pointer alignment the kernel needs is not met           */
#define TB_ELAUNCH (-3)  /* the CUDA launch (or a CUDA runtime call) failed         */
#define TB_EDEVICE (-4)  /* the current device is not sm_100 / has no usable kernel */

/* Text of the last error reported on this host thread ("" when none). */
const char *tb_last_error(void);

/* Library version, (major << 16) | (minor << 8) | patch. */
int tb_version(void);

/* Bounded waits (on mbarriers of bulk copies) that gave up on `device` (-1: the current one)
 * since the library was loaded; each such kernel returned early instead of hanging, so a
 * nonzero count means its output is incomplete. Synchronising. No counterpart in the
 * reference (its Triton kernels do not wait on barriers). */
int tb_wait_timeouts(int32_t device, uint32_t *count);

/* Self-test of the bounded wait behind tb_wait_timeouts: one thread waits on phase 0 of an
 * mbarrier in its own shared memory (expecting one arrival) for at most `polls` polls, after
 * arriving on it itself when `arrive` is nonzero. *status (device int32) = 0 when the phase
 * completed, 1 when the wait gave up, which also adds 1 to tb_wait_timeouts. Shows that a wait
 * that runs out returns an error status and leaves the context usable. No counterpart in the
 * reference (its Triton kernels wait on no barriers). */
int tb_wait_selftest(int32_t polls, int32_t arrive, int32_t *status, void *stream);

/* Kernel launches this library has queued since it was loaded, all threads and devices (a
 * launch captured into a CUDA graph counts once, when captured). No reference counterpart. */
int64_t tb_launch_count(void);

/* ---------------------------------------------------------------------------------------------
 * NF4 unpack (bitsandbytes 4-bit layout). Replaces nf4_unpack_kernel and its launch in
 * unpack_into, solution/nf4.py:27-45 and :72-89.
 *
 *   nested:  absmax[b] = fp32(code2[absmax_u8[b]] * absmax2[b / qblock2]) + offset[0]
 *   plain:   absmax[b] = absmax_f32[b]
 *   out[2j]   = fp16(nf4[packed[j] >> 4]  * absmax[(2j) / qblock])   (high nibble first)
 *   out[2j+1] = fp16(nf4[packed[j] & 15] * absmax[(2j) / qblock])
 * Each product and sum is rounded on its own (no FMA), then rounded once to fp16, so the output
 * is bit-exact with the reference for the same 16-entry nf4 table.
 * qblock must be even; n_bytes counts packed bytes (= values / 2).
 * ------------------------------------------------------------------------------------------- */
int tb_nf4_unpack_nested(const uint8_t *packed, const uint8_t *absmax_u8, const float *code2,
                         const float *absmax2, const float *offset, const float *nf4_table,
                         uint16_t *out, int64_t n_bytes, int32_t qblock, int32_t qblock2,
                         void *stream);

int tb_nf4_unpack_plain(const uint8_t *packed, const float *absmax, const float *nf4_table,
                        uint16_t *out, int64_t n_bytes, int32_t qblock, void *stream);

/* One launch for up to TB_NF4_MAX_WEIGHTS weights (for example q|k|v or gate|up stacked into
 * one GEMM operand). Replaces the per-weight loop of unpack_concat, solution/nf4.py:96-105.
 * Arrays are HOST arrays of length n_weights. For weight i: absmax_f32[i] non-NULL selects the
 * plain layout, else the nested fields (absmax_u8, code2, absmax2, offset, qblock2) are used. */
#define TB_NF4_MAX_WEIGHTS 8
int tb_nf4_unpack_multi(int32_t n_weights, const uint8_t *const *packed,
                        const float *const *absmax_f32, const uint8_t *const *absmax_u8,
                        const float *const *code2, const float *const *absmax2,
                        const float *const *offset, const float *const *nf4_table,
                        uint16_t *const *out, const int64_t *n_bytes, const int32_t *qblock,
                        const int32_t *qblock2, void *stream);

/* ---------------------------------------------------------------------------------------------
 * NF4-weight GEMMs on the tensor cores (tcgen05, TMEM accumulator, TMA token tiles) with the NF4
 * decode in the operand producer: the fp16 copy of the frozen weight is never written. Replaces
 * FrozenNF4Linear (unpack + cuBLAS in both directions, solution/nf4.py:108-127) and the unpack +
 * GEMMs of FusedNF4MLP (solution/mlp.py:80-113).
 *
 * W is 1..TB_NF4_GEMM_MAX_WEIGHTS weights stacked by rows (q|k|v, gate|up), each in
 * bitsandbytes' packing (row-major [rows[j], k_dim], blocksize 64, high nibble first) with its
 * fp32 absmax per block given block-column-major: absmax_t[j] is [k_dim / 64, rows[j]] (a nested
 * state's absmax expanded by the caller: fp32(code2[c] * absmax2[b / 256]) + offset, each
 * operation rounded on its own). Every decoded value is fp16(table[q] * absmax), bit-identical
 * to tb_nf4_unpack_*; the products differ from cuBLAS over the unpacked weight only in the order
 * of the fp32 sums.
 *   transpose 0: out[t, n] = fp16(sum_k in[t, k] W[n, k] (+ bias[n]))   in [tokens, k_dim]
 *                rows[j] multiples of 128, k_dim of 64
 *   transpose 1: out[t, k] = fp16(sum_n in[t, n] W[n, k])               in [tokens, sum rows]
 *                rows[j] multiples of 64, k_dim of 128, no bias
 * Arrays packed / absmax_t / nf4_table / rows are HOST arrays of length n_weights. Row strides
 * ld_in / ld_out in elements, multiples of 8; in, out, bias, packed, absmax_t 16-byte aligned.
 * Persistent CTAs run the (128-row tile, token group, reduction split) units; when the reduction
 * is split the fp32 partials go to `workspace` (tb_nf4_gemm_workspace bytes; without it the
 * reduction is not split) and are summed in split order. sm_100 only.
 * ------------------------------------------------------------------------------------------- */
#define TB_NF4_GEMM_MAX_WEIGHTS 4
int tb_nf4_gemm(int32_t transpose, const uint16_t *tokens_in, int64_t tokens, int64_t ld_in,
                int32_t n_weights, const uint8_t *const *packed, const float *const *absmax_t,
                const float *const *nf4_table, const int64_t *rows, int64_t k_dim,
                const uint16_t *bias, uint16_t *out, int64_t ld_out, float *workspace,
                int64_t workspace_bytes, void *stream);

/* Bytes of fp32 workspace tb_nf4_gemm needs for these shapes under the current variant (0 when
 * the reduction is not split). No counterpart in the reference. */
int64_t tb_nf4_gemm_workspace(int32_t transpose, int64_t tokens, int32_t n_weights,
                              const int64_t *rows, int64_t k_dim);

/* How tb_nf4_gemm plans the reduction, process-wide: 0 split so that the work units fill the GPU
 * (fp32 partials in the workspace), 1 never split. Same results either way (up to the order of
 * the fp32 sums). No counterpart in the reference. */
int tb_nf4_gemm_variant(int32_t variant);

/* The MLP's NF4 GEMMs with SwiGLU in the epilogue (solution/mlp.py:31-58 applied to the GEMM's
 * fp16 output, solution/mlp.py:82-113):
 *   backward 0: weights (gate, up), each [inter, k_dim]; tokens_in = x [tokens, k_dim]; writes
 *               gu = fp16(x [gate|up]^T) [tokens, 2 inter] (row stride ld_gu) and
 *               act = fp16(silu(g) u) [tokens, inter] (row stride ld_act)
 *   backward 1: weight (down,) [hidden, inter] (k_dim = inter); tokens_in = dy [tokens, hidden];
 *               dact = fp16(dy . W_down) stays in the epilogue, which overwrites gu in place
 *               with d(gate|up) (act unused, may be NULL). */
int tb_nf4_gemm_swiglu(int32_t backward, const uint16_t *tokens_in, int64_t tokens, int64_t ld_in,
                       int32_t n_weights, const uint8_t *const *packed,
                       const float *const *absmax_t, const float *const *nf4_table,
                       const int64_t *rows, int64_t k_dim, uint16_t *gu, int64_t ld_gu,
                       uint16_t *act, int64_t ld_act, void *stream);

/* The q|k|v projection with its bias, the LoRA rows and the rotary embedding: weights (q, k, v) =
 * [n_heads * 128, k_dim], [n_kv * 128, k_dim] twice (HOST arrays of 3); x fp16 [tokens, k_dim]
 * (row stride ld_x); bias fp16 [(n_heads + 2 n_kv) * 128] or NULL; lora_q fp16
 * [tokens, n_heads * 128], lora_v fp16 [tokens, n_kv * 128] or NULL; cos, sin fp32 [seq, 128];
 * pos_idx int64 [tokens] padded positions (t = pos % seq; a negative position writes nothing).
 * Writes token-major q [tokens, n_heads, 128], k, v [tokens, n_kv, 128]: what
 * tb_rope_tokens_fwd writes from the GEMM's fp16 output (solution/rope.py:24-75 with the padded
 * scatter replaced by token-major rows). The GEMM's fp32 partials go to `workspace`
 * (tb_nf4_gemm_qkv_rope_workspace bytes, 16-byte aligned); a second kernel finishes them. */
int tb_nf4_gemm_qkv_rope(const uint16_t *x, int64_t tokens, int64_t ld_x,
                         const uint8_t *const *packed, const float *const *absmax_t,
                         const float *const *nf4_table, int64_t k_dim, const uint16_t *bias,
                         const uint16_t *lora_q, const uint16_t *lora_v, const float *cos,
                         const float *sin, const int64_t *pos_idx, int64_t seq, int32_t n_heads,
                         int32_t n_kv, uint16_t *q, uint16_t *k, uint16_t *v, float *workspace,
                         int64_t workspace_bytes, void *stream);

/* Bytes of workspace tb_nf4_gemm_qkv_rope needs. No counterpart in the reference. */
int64_t tb_nf4_gemm_qkv_rope_workspace(int64_t tokens, int32_t n_heads, int32_t n_kv,
                                       int64_t k_dim);

/* ---------------------------------------------------------------------------------------------
 * Residual add + RMSNorm. Replaces rmsnorm_fwd_kernel / rmsnorm_bwd_kernel and their launches,
 * solution/rmsnorm.py:24-69 and :76-112.
 *
 * forward, per row r of [rows, hidden]:
 *   s = x (+ delta)           fp32, written to s_out only when delta != NULL
 *   rstd = 1 / sqrt(sum(s*s) / hidden + eps)
 *   y = fp16((s * rstd) * weight);  ypad[pad_idx[r]] = fp32 value of the same product
 *   rstd_out[r] = rstd
 * x fp32, delta fp16 (nullable), weight fp32, ypad fp32 [padded_rows, hidden] (nullable, together
 * with pad_idx int64 [rows]). ypad rows that no pad_idx names are NOT touched (zero them first).
 * ------------------------------------------------------------------------------------------- */
int tb_add_rmsnorm_fwd(const float *x, const uint16_t *delta, const float *weight, float *s_out,
                       uint16_t *y, float *ypad, const int64_t *pad_idx, float *rstd_out,
                       int64_t rows, int64_t hidden, float eps, void *stream);

/* backward, per row r:
 *   g = (dy (+ dypad[pad_idx[r]])) * weight        dy fp16, dypad fp32; either may be NULL
 *   n = s * rstd
 *   dx = (g - n * sum(g*n) / hidden) * rstd (+ ds)  fp32 out; ddelta = fp16(dx) when non-NULL */
int tb_add_rmsnorm_bwd(const float *s, const float *rstd, const float *weight, const uint16_t *dy,
                       const float *dypad, const int64_t *pad_idx, const float *ds, float *dx,
                       uint16_t *ddelta, int64_t rows, int64_t hidden, void *stream);

/* The same backward (no padded gradient) with dy given as the fp32 K-split partial products of
 * the GEMM that produces it (the MLP's gate|up backward, K = 2 x intermediate, as one batched
 * GEMM): n_parts arrays [rows, hidden] part_stride elements apart, summed in part order and
 * rounded to fp16 once (the GEMM's fp16 output), so no split-K reduce launch runs. hidden a
 * multiple of 8 and every buffer 16-byte aligned (TB_EINVAL / TB_EALIGN otherwise). */
int tb_add_rmsnorm_bwd_parts(const float *s, const float *rstd, const float *weight,
                             const float *dy_parts, int32_t n_parts, int64_t part_stride,
                             const float *ds, float *dx, uint16_t *ddelta, int64_t rows,
                             int64_t hidden, void *stream);

/* The same backward with dypad formed in registers from the rank-16 LoRA pair the padded output
 * feeds (solution/model.py:195-206 under fp16 autocast: the dropout backward of lora_A's input
 * gradient), instead of read from a tensor tb_lora_dropout_grad_expand wrote: per row r, slot
 * p = pad_idx[r] and column c,
 *   dypad[p, c] = drop_q'(fp16(dh_q[r] . a16_q[:, c])) + drop_v'(fp16(dh_v[r] . a16_v[:, c]))
 *   drop'(x) = mask[p, c] ? x * scale : 0 (x when mask is NULL)
 * with tb_lora_dropout_grad_expand's operations and roundings, and tb_add_rmsnorm_bwd's arithmetic
 * after it. The outputs equal that two-launch path's bit for bit wherever tb_add_rmsnorm_bwd
 * plans one or two 8-column chunks per thread (for 1536 columns: up to 1381 rows); where it plans
 * more for a large row count, its row sums run in another order and agree to fp32 rounding.
 * dh: fp16 [rows, 16]; a16: fp16 [16, hidden]; mask: bool [slots, hidden]; an adapter with dh
 * NULL is absent. rank must be 16 and hidden a multiple of 8 up to 4096 (TB_EINVAL otherwise);
 * all buffers 16-byte aligned, masks 8-byte (TB_EALIGN). */
int tb_add_rmsnorm_bwd_lora(const float *s, const float *rstd, const float *weight,
                            const uint16_t *dy, const int64_t *pad_idx, const float *ds,
                            const uint16_t *dh_q, const uint16_t *a16_q, const uint8_t *mask_q,
                            float scale_q, const uint16_t *dh_v, const uint16_t *a16_v,
                            const uint8_t *mask_v, float scale_v, float *dx, uint16_t *ddelta,
                            int64_t rows, int64_t hidden, int32_t rank, void *stream);

/* ---------------------------------------------------------------------------------------------
 * QKV pack: LoRA add + rotary embedding + scatter into the padded attention layout. Replaces
 * rope_pack_fwd_kernel / rope_pack_bwd_kernel and RopePack, solution/rope.py:24-128, :136-176.
 *
 * qkv fp16 [rows, (nh + 2 nkv) * d]; lora_q [rows, nh*d] and lora_v [rows, nkv*d] (nullable;
 * lora_is_fp32 selects fp32, else fp16); cos/sin fp32 [seq, d]; pos_idx int64 [rows] (padded
 * position b*seq + t of each token). Outputs q fp16 [batch, nh, seq, d], k/v [batch, nkv, seq, d].
 *   q = rot(qkv_q + lq), k = rot(qkv_k), v = qkv_v + lv, rot(x)=(x1 c1 - x2 s1, x2 c2 + x1 s2)
 * slot_tok (nullable) is int32 [batch*seq]: the token at each padded slot or -1. When given, the
 * kernel covers every slot and writes the zero rows itself; when NULL it writes only the token
 * rows and the caller must have zeroed q, k, v.
 * ------------------------------------------------------------------------------------------- */
int tb_rope_pack_fwd(const uint16_t *qkv, const void *lora_q, const void *lora_v,
                     int32_t lora_is_fp32, const float *cos, const float *sin,
                     const int64_t *pos_idx, const int32_t *slot_tok, uint16_t *q, uint16_t *k,
                     uint16_t *v, int64_t rows, int64_t batch, int64_t seq, int32_t n_heads,
                     int32_t n_kv, int32_t head_dim, void *stream);

/* dqkv fp16 [rows, (nh + 2 nkv) * d] from dq/dk/dv fp16 in the padded layout (each nullable =
 * zero gradient): inverse rotation (g1 c1 + g2 s2, g2 c2 - g1 s1) for q and k, copy for v. */
int tb_rope_pack_bwd(const uint16_t *dq, const uint16_t *dk, const uint16_t *dv, const float *cos,
                     const float *sin, const int64_t *pos_idx, uint16_t *dqkv, int64_t rows,
                     int64_t batch, int64_t seq, int32_t n_heads, int32_t n_kv, int32_t head_dim,
                     void *stream);

/* The same QKV pack with token-major outputs: q fp16 [rows, nh, d], k and v [rows, nkv, d], the
 * packed layout of variable-length attention (cumulative sequence offsets instead of padding);
 * pos_idx still gives each token's position b*seq + t (its rotary row t). No padded slot is
 * written. No counterpart in the reference, whose attention runs on the padded layout
 * (solution/model.py:242-246). */
int tb_rope_tokens_fwd(const uint16_t *qkv, const void *lora_q, const void *lora_v,
                       int32_t lora_is_fp32, const float *cos, const float *sin,
                       const int64_t *pos_idx, uint16_t *q, uint16_t *k, uint16_t *v,
                       int64_t rows, int64_t batch, int64_t seq, int32_t n_heads, int32_t n_kv,
                       int32_t head_dim, void *stream);

/* Backward of tb_rope_tokens_fwd: dqkv fp16 [rows, (nh + 2 nkv) * d] from token-major dq, dk,
 * dv (each nullable = zero gradient). */
int tb_rope_tokens_bwd(const uint16_t *dq, const uint16_t *dk, const uint16_t *dv,
                       const float *cos, const float *sin, const int64_t *pos_idx,
                       uint16_t *dqkv, int64_t rows, int64_t batch, int64_t seq, int32_t n_heads,
                       int32_t n_kv, int32_t head_dim, void *stream);

/* slot_tok[b*seq+t] = token index at that padded slot, -1 for padding (the inverse of pos_idx).
 * Helper for tb_rope_pack_fwd; a memset plus one scatter kernel. */
int tb_slot_index(const int64_t *pos_idx, int64_t rows, int64_t slots, int32_t *slot_tok,
                  void *stream);

/* ---------------------------------------------------------------------------------------------
 * LoRA branches of q_proj / v_proj around PyTorch's dropout (the reference's _lora_branch,
 * solution/model.py:195-206: lora_B(lora_A(dropout(x_pad))) * scaling on the real tokens; no
 * kernel of its own there: index_select, casts, index_add and dropout backward in PyTorch).
 * ------------------------------------------------------------------------------------------- */

/* x16[r] = fp16(dropped[pos_idx[r]]) for each of q and v (either pair nullable): the real rows of
 * the fp32 dropout outputs [slots, hidden] gathered and cast to fp16 [rows, hidden], the input
 * lora_A reads under fp16 autocast. */
int tb_lora_gather(const float *dropped_q, const float *dropped_v, const int64_t *pos_idx,
                   uint16_t *xq, uint16_t *xv, int64_t rows, int64_t hidden, void *stream);

/* Both adapters' forward for rank-16 LoRA, per real row m (either adapter's weights NULL when
 * absent): x16[m] = fp16(dropped[pos_idx[m]]); h16[m] = fp16(x16[m] . fp16(a)^T);
 * out[m] = fp16(fp32(fp16(h16[m] . fp16(b)^T)) * scale), fp32 accumulation on the tensor cores.
 * dropped: fp32 [slots, hidden] dropout outputs; a: lora_A weight fp32 [16, hidden]; b: lora_B
 * weight fp32 [hout, 16]; a16 / b16: their fp16 casts, written here for the backward GEMMs; x16
 * [rows, hidden], h16 [rows, 16] (kept for backward), out [rows, hout], fp16. hidden a multiple
 * of 16, hout of 8. Replaces lora_A, lora_B and "* scaling" under fp16 autocast with their
 * weight casts (peft, called from solution/model.py:205), and the index_select + cast of
 * tb_lora_gather. */
int tb_lora_forward(const float *dropped_q, const float *a_q, const float *b_q, uint16_t *a16_q,
                    uint16_t *b16_q, uint16_t *x16_q, uint16_t *h16_q, uint16_t *out_q,
                    int64_t hout_q, float scale_q, const float *dropped_v, const float *a_v,
                    const float *b_v, uint16_t *a16_v, uint16_t *b16_v, uint16_t *x16_v,
                    uint16_t *h16_v, uint16_t *out_v, int64_t hout_v, float scale_v,
                    const int64_t *pos_idx, int64_t rows, int64_t hidden, int32_t rank,
                    void *stream);

/* The padded gradient of the dropout input both adapters share, fp32 [slots, hidden]:
 * grad[p] = fp32(dxq[t]) * scale_q * mask_q[p] + fp32(dxv[t]) * scale_v * mask_v[p] for the token
 * t = slot_tok[p], 0 where slot_tok[p] < 0. dxq / dxv: fp16 [rows, hidden] gradients of the fp16
 * lora_A inputs (nullable: that adapter is absent); mask_q / mask_v: the dropout keep masks
 * (bool bytes [slots, hidden]; nullable: no dropout, the gradient passes unscaled); scale =
 * 1 / (1 - p) as the dropout backward takes it. Each product and the sum rounded on its own. */
int tb_lora_dropout_grad(const uint16_t *dxq, const uint16_t *dxv, const uint8_t *mask_q,
                         const uint8_t *mask_v, const int32_t *slot_tok, float *grad,
                         int64_t slots, int64_t hidden, float scale_q, float scale_v,
                         void *stream);

/* tb_lora_dropout_grad with the adapters' lora_A input gradients computed inside it: for rank 16,
 * dx = fp16(dh . a16) (dh fp16 [rows, 16], a16 = fp16(lora_A) [16, hidden], fp32 sums in rank
 * order, as the fp16 GEMM `dh @ a16` under autocast gives it) for each adapter, then the same
 * dropout backward and sum into grad fp32 [slots, hidden] (0 at padding slots). Replaces the
 * two dx GEMMs and the dropout backward of _lora_branch's backward (solution/model.py:195-206).
 * hidden a multiple of 8; 16-byte aligned dh, a16 and grad. Either adapter may be absent (NULL
 * dh). */
int tb_lora_dropout_grad_expand(const uint16_t *dh_q, const uint16_t *a16_q, const uint16_t *dh_v,
                                const uint16_t *a16_v, const uint8_t *mask_q,
                                const uint8_t *mask_v, const int32_t *slot_tok, float *grad,
                                int64_t slots, int64_t hidden, int32_t rank, float scale_q,
                                float scale_v, void *stream);

/* The rank-16 LoRA backward of both adapters (q, then v; an adapter whose g is NULL is skipped)
 * in two launches, in place of the six cuBLAS GEMMs of peft's lora_B(lora_A(x)) * scaling
 * backward under fp16 autocast (solution/model.py:195-206). Per adapter: g fp16 [rows, width]
 * with row stride ld_g_q / ld_g_v (>= width, a multiple of 8: the output gradient, for example
 * the adapter's columns of the q|k|v gradient, read in place), h fp16 [rows, 16] (lora_A's output), b16 = fp16(lora_B) [width, 16],
 * x16 fp16 [rows, hidden] (lora_A's input):
 *   dh = fp16(scale * g . b16)    [rows, 16] fp16
 *   db = scale * g^T . h          [width, 16] fp32 (added into db when its accumulate bit is set)
 *   da = dh^T . x16               [16, hidden] fp32 (added into da when its accumulate bit is set)
 * accumulate: bit 0 db_q, bit 1 da_q, bit 2 db_v, bit 3 da_v. rank must be 16; width and hidden
 * multiples of 64; g, h, b16, x16, dh 16-byte aligned. Sums in a fixed order (deterministic).
 * Two launches: dh and db on `stream`, then da. With stream_da non-NULL (and not `stream`), da
 * runs on stream_da after an event recorded on `stream` behind the first launch, beside what the
 * caller queues next on `stream`; the caller makes `stream` wait for stream_da before reading
 * da. */
int tb_lora_backward(const uint16_t *g_q, const uint16_t *h_q, const uint16_t *b16_q,
                     const uint16_t *x16_q, uint16_t *dh_q, float *db_q, float *da_q,
                     int64_t width_q, float scale_q, const uint16_t *g_v, const uint16_t *h_v,
                     const uint16_t *b16_v, const uint16_t *x16_v, uint16_t *dh_v, float *db_v,
                     float *da_v, int64_t width_v, float scale_v, int64_t rows, int64_t hidden,
                     int32_t rank, int32_t accumulate, int64_t ld_g_q, int64_t ld_g_v,
                     void *stream, void *stream_da);

/* ---------------------------------------------------------------------------------------------
 * Causal attention over packed variable-length sequences with grouped key/value heads. Replaces
 * the decoder layer's SDPA over the padded layout (solution/model.py:242-247) for the real rows:
 * q fp16 [total, n_heads, head_dim], k, v fp16 [total, n_kv, head_dim] (token-major, the
 * sequences packed back to back), cu_seqlens int32 [batch + 1] (sequence b holds tokens
 * cu[b] .. cu[b+1]-1, no longer than max_len); query i of a sequence attends to its keys 0..i;
 * query head h uses key/value head h / (n_heads / n_kv). head_dim 128.
 * tb_attn_varlen_fwd: out fp16 [total, n_heads, head_dim] = softmax(scale q k^T) v, and
 *   lse fp32 [n_heads, total], the base-2 log-sum-exp of scale * log2(e) * q k^T per query (what
 *   the backward recomputes the probabilities from).
 * ------------------------------------------------------------------------------------------- */
int tb_attn_varlen_fwd(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                       const int32_t *cu_seqlens, uint16_t *out, float *lse, int64_t batch,
                       int64_t total, int64_t max_len, int32_t n_heads, int32_t n_kv,
                       int32_t head_dim, float scale, void *stream);

/* tb_attn_varlen_fwd on the 5th-generation tensor cores (same arguments, outputs and
 * tolerances): a CTA per 128 queries of a head of a sequence; S = q k^T and O = P v accumulate
 * in tensor memory (tcgen05.mma, q / k / v tiles by TMA), P is written to tensor memory as the
 * A operand of P v; one pass over the key tiles with the next tile's scores computed while the
 * current one's softmax runs, and O rescaled in tensor memory only when a row's maximum grows by
 * more than 2^8. sm_100 only; q, k, v, out 16-byte aligned. Replaces the same SDPA call,
 * solution/model.py:242-247. */
int tb_attn_varlen_fwd_tc(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                          const int32_t *cu_seqlens, uint16_t *out, float *lse, int64_t batch,
                          int64_t total, int64_t max_len, int32_t n_heads, int32_t n_kv,
                          int32_t head_dim, float scale, void *stream);

/* tb_attn_varlen_bwd: from the forward's q, k, v, out, lse and the output gradient dout
 *   (fp16 [total, n_heads, head_dim]): dq fp16 [total, n_heads, head_dim], dk, dv fp16
 *   [total, n_kv, head_dim] (the query heads of a group summed in head order in fp32, rounded
 *   once). Scratch the caller provides: delta fp32 [n_heads, total] (rowsum(dout o out)),
 *   dk_part, dv_part fp32 [total, n_heads, head_dim] (per-query-head partials). Deterministic. */
int tb_attn_varlen_bwd(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                       const uint16_t *out, const uint16_t *dout, const float *lse,
                       const int32_t *cu_seqlens, uint16_t *dq, uint16_t *dk, uint16_t *dv,
                       float *delta, float *dk_part, float *dv_part, int64_t batch, int64_t total,
                       int64_t max_len, int32_t n_heads, int32_t n_kv, int32_t head_dim,
                       float scale, void *stream);

/* tb_attn_varlen_bwd whose gradients leave through the rotary embedding's backward: instead of
 * dq, dk, dv it writes dqkv fp16 [total, (n_heads + 2 n_kv) * 128] (row stride ld_qkv) =
 * [rot^-1(dq) | rot^-1(dk) | dv] per token, what tb_rope_tokens_bwd writes from those fp16
 * gradients (solution/rope.py:78-128, token-major): each gradient rounded to fp16, then
 * (g1 c1 + g2 s2, g2 c2 - g1 s1) with cos, sin fp32 [seq, 128] at t = pos_idx[token] % seq; a
 * position outside [0, slots) gives a zero row. No dq / dk / dv tensors are materialised: the
 * dQ kernel writes fp16 dQ into dqkv's q columns, and the last kernel of the call rotates those
 * in place while it sums, rotates and writes the key/value gradients. cos and sin must be
 * 16-byte aligned. */
int tb_attn_varlen_bwd_rope(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                            const uint16_t *out, const uint16_t *dout, const float *lse,
                            const int32_t *cu_seqlens, const float *cos, const float *sin,
                            const int64_t *pos_idx, int64_t seq, int64_t slots, uint16_t *dqkv,
                            int64_t ld_qkv, float *delta, float *dk_part, float *dv_part,
                            int64_t batch, int64_t total, int64_t max_len, int32_t n_heads,
                            int32_t n_kv, int32_t head_dim, float scale, void *stream);

/* ---------------------------------------------------------------------------------------------
 * Gated SiLU. Replaces gated_silu_fwd_kernel / gated_silu_bwd_inplace_kernel,
 * solution/mlp.py:31-58 and :61-77.
 *   gu fp16 [rows, 2*inter] = [gate | up];  act = fp16(gate / (1 + exp(-gate)) * up)
 *   backward, IN PLACE over gu:  sig = 1/(1+exp(-g));  [g | u] <- [dact*u*sig*(1+g(1-sig)) |
 *   dact*(g*sig)], dact fp16 [rows, inter].
 * ------------------------------------------------------------------------------------------- */
int tb_swiglu_fwd(const uint16_t *gu, uint16_t *act, int64_t rows, int64_t inter, void *stream);
int tb_swiglu_bwd_inplace(const uint16_t *dact, uint16_t *gu, int64_t rows, int64_t inter,
                          void *stream);

/* ---------------------------------------------------------------------------------------------
 * Vocabulary head statistics over a chunk of fp16 logits, IN PLACE. Replaces
 * head_stats_grad_kernel, solution/head.py:34-76 (launch :108-110).
 * logits fp16 [rows, vocab] with row stride ld (elements); targets int64 [rows] (-100 = none).
 * Per row: lse, entropy = lse - sum(p z), loss = lse - z[target] (0 when unlabelled),
 * correct = labelled & (first argmax == target); for labelled rows the logits are overwritten
 * with fp16((exp(z - lse) - onehot) * grad_scale). Targets outside [0, vocab) other than -100
 * are an error the caller must rule out (the row is then treated as unlabelled).
 * ------------------------------------------------------------------------------------------- */
int tb_head_stats_grad(uint16_t *logits, const int64_t *targets, float *entropy, float *loss,
                       int32_t *correct, int64_t rows, int64_t vocab, int64_t ld,
                       float grad_scale, void *stream);

/* Split form of the same statistics, for rows spread over several CTAs or several GPUs (a
 * vocabulary-sharded head). No counterpart kernel in the reference, whose one launch per chunk
 * covers whole rows (solution/head.py:34-76); these three compute the same values.
 *
 * tb_head_partials: logits fp16 [rows, cols] (row stride ld) hold vocabulary columns
 * col_offset .. col_offset+cols-1. Each row is cut into `splits` column ranges; for each range:
 *   part fp32 [rows, splits, 6] = (max z, sum e^(z-max), sum e^(z-max) z, best z,
 *                                  z[target] if the target column is in the range else 0,
 *                                  1 if it is else 0)
 *   part_idx int64 [rows, splits] = vocabulary index of the first maximum in the range.
 * rows <= 65535 per call. */
int tb_head_partials(const uint16_t *logits, const int64_t *targets, float *part,
                     int64_t *part_idx, int64_t rows, int64_t cols, int64_t ld,
                     int64_t col_offset, int32_t splits, void *stream);

/* Merges n_groups x splits partial states per row, laid out [group][row][split] (for example the
 * partials of every rank, gathered): lse, entropy = lse - sum(p z), loss = lse - z[target]
 * (0 for unlabelled rows) and correct = first argmax == target. */
int tb_head_merge(const float *part, const int64_t *part_idx, const int64_t *targets,
                  int64_t rows, int32_t n_groups, int32_t splits, float *lse, float *entropy,
                  float *loss, int32_t *correct, void *stream);

/* The head's labelled-first row order (the gather of labelled rows in solution/head.py:87-156,
 * as a stable partition): order[i] is the row at sorted place i, labelled rows (target !=
 * ignore_index) first, each group in row order; targets_sorted[i] = targets[order[i]]. One
 * launch (one CTA), no host synchronisation. */
/* The token embedding of the real tokens: out[r] = fp32(table[ids[pos_idx[r]]]) (the fused path
 * of solution/model.py:220-225: index_select of the ids, the embedding gather and the cast to the
 * fp32 residual stream in one launch). ids int64 [slots] (the padded batch, flattened); table
 * fp16 [vocab, hidden], hidden a multiple of 8, table and out 16-byte aligned. An id outside
 * [0, vocab) reads nothing: its row is written as zeros and counted (tb_embed_invalid_ids). */
int tb_embed_rows(const int64_t *ids, const int64_t *pos_idx, const uint16_t *table, float *out,
                  int64_t rows, int64_t hidden, int64_t vocab, void *stream);

/* Token ids tb_embed_rows found outside [0, vocab) since the library was loaded (-1 when the
 * counter cannot be read). */
int64_t tb_embed_invalid_ids(void);

int tb_head_order(const int64_t *targets, int64_t rows, int64_t ignore_index, int64_t *order,
                  int64_t *targets_sorted, void *stream);

/* Back to row order after the head: grad[order[i]] = dh_sorted[i] for i < keep and 0 for the
 * other rows (fp16 [rows, width], width a multiple of 8, 16-byte aligned; grad NULL: statistics
 * only), entropy[order[i]] = entropy_sorted[i], loss likewise, correct[order[i]] =
 * (correct_sorted[i] != 0) as bytes. Replaces the zero fill + index_copy of the gradient and the
 * inverse permutation + gathers of the statistics (solution/head.py:113-156). */
int tb_head_unsort(const int64_t *order, int64_t rows, int64_t keep, const uint16_t *dh_sorted,
                   int64_t width, uint16_t *grad, const float *entropy_sorted,
                   const float *loss_sorted, const int32_t *correct_sorted, float *entropy,
                   float *loss, uint8_t *correct, void *stream);

/* Folds partial states: for each row, its splits_in states (part [rows, splits_in, 6],
 * part_idx [rows, splits_in], the layout tb_head_partials and tb_head_logits_stats write) are
 * merged in splits_out contiguous groups into part_out [rows, splits_out, 6] and idx_out
 * [rows, splits_out], every argmax index shifted by col_offset. A vocabulary shard folds its
 * per-tile states to one per row (indices made global with its first column) before the
 * exchange between GPUs; tb_head_merge of the folded states gives what it gives unfolded. No
 * counterpart in the reference (its head is one GPU, solution/head.py:54-72 merges inside one
 * kernel). */
int tb_head_fold(const float *part, const int64_t *part_idx, int64_t rows, int32_t splits_in,
                 int64_t col_offset, int32_t splits_out, float *part_out, int64_t *idx_out,
                 void *stream);

/* The head's logits GEMM on the tensor cores with sweep 1 fused into its epilogue. For rows of
 * hidden fp16 [rows, hidden_dim] and the head weight fp16 [vocab, hidden_dim] (both row-major,
 * hidden_dim a multiple of 64, 16-byte aligned): z = fp16(hidden . weight^T) (tcgen05.mma, fp32
 * accumulation in TMEM, rounded to fp16 as the reference's fp16 GEMM output,
 * solution/head.py:107) and, per row and 256-column vocabulary tile, the partial state of
 * tb_head_partials: part fp32 [rows, ceil(vocab/256), 6], part_idx int64 [rows, ceil(vocab/256)]
 * (merge them with tb_head_merge, n_groups 1, splits ceil(vocab/256)). When logits is non-NULL
 * the fp16 logits of the first logits_rows rows are written to it ([logits_rows, vocab]) for
 * the dlogits pass. A target outside [0, vocab) (IGNORE_INDEX, or on a vocabulary shard a
 * label another shard holds, passed as -1) matches no column. Replaces the cuBLAS logits GEMM +
 * sweep 1 of the reference's head (solution/head.py:107-110, :54-72). sm_100 only. */
int tb_head_logits_stats(const uint16_t *hidden, const uint16_t *weight, const int64_t *targets,
                         uint16_t *logits, int64_t logits_rows, float *part, int64_t *part_idx,
                         int64_t rows, int64_t vocab, int64_t hidden_dim, void *stream);

/* Which tensor-core kernel tb_head_logits_stats uses, process-wide: 0 automatic, 1 the 1-SM
 * kernel (128x256 tiles, tcgen05.mma.cta_group::1), 2 the 2-SM kernel (256x256 tiles per CTA
 * pair, tcgen05.mma.cta_group::2). Same results either way. No counterpart in the reference. */
int tb_head_gemm_variant(int32_t variant);

/* tb_head_stats_grad's contract (the same outputs, the same in-place dlogits) with nothing
 * allocated anywhere, for callers that cannot allocate device memory themselves: a host binding
 * that only ever receives buffers owned by someone else (a plain C FFI from another language
 * runtime), a process whose framework allocator has reserved all device memory so that a
 * cudaMalloc here would fail or fragment it, or a latency-critical loop that cannot afford the
 * device synchronisation cudaMalloc implies. No counterpart in the reference (its head kernel,
 * solution/head.py:34-76, needs no scratch). The scratch it uses (partial states of the split
 * form, 1,179,648 bytes) is a fixed array inside the library: each GPU that loads the library
 * holds it until the process exits. At most 32768 rows per call (larger calls are rejected with
 * TB_EINVAL). Outside stream capture each call looks up the array's device address; during
 * capture the address an earlier call on that device took is used, so make the first call on
 * a device before any stream capture (a first call inside capture is rejected). Calls share the
 * array: calls whose kernels overlap on the GPU (different streams, no ordering) race and must
 * not be made. */
int tb_head_stats_grad_noalloc(uint16_t *logits, const int64_t *targets, float *entropy,
                               float *loss, int32_t *correct, int64_t rows, int64_t vocab,
                               int64_t ld, float grad_scale, void *stream);

/* The head's hidden-state gradient with the logits gradient formed inside the tensor-core GEMM
 * (replaces the in-place dlogits of solution/head.py:73-76 followed by the cuBLAS
 * dh_chunk = dlogits[:lab] @ W of solution/head.py:113). For the first `rows` rows of the fp16
 * logits slab [rows, cols] (row stride ld, columns col_offset .. of the vocabulary) with lse fp32
 * [rows] and targets int64 [rows] (global columns; IGNORE_INDEX rows give a zero gradient):
 *   dl[r, c] = fp16((e^(z[r, c] - lse[r]) - [col_offset + c == targets[r]]) * grad_scale)
 *              (bit-identical to what tb_head_dlogits writes; never stored)
 *   dh[r, :] = sum_c dl[r, c] W[c, :]     W fp16 [cols, hidden_dim], fp32 accumulation
 * written to out row out_rows[r] (out_rows NULL: row r), row stride ld_out: fp32 when out_fp32
 * (added to what out holds when accumulate is set), else rounded to fp16. The vocabulary is
 * split over CTAs; their fp32 partials go to `workspace` (tb_head_dh_workspace bytes, 16-byte
 * aligned) and are summed in a fixed order (deterministic). hidden_dim a multiple of 256, ld a
 * multiple of 8, ld_out of 4; logits, weight, workspace 16-byte aligned. sm_100 only. */
int tb_head_dh(const uint16_t *logits, int64_t ld, const int64_t *targets, const float *lse,
               int64_t rows, int64_t cols, int64_t col_offset, float grad_scale,
               const uint16_t *weight, int64_t hidden_dim, float *workspace,
               int64_t workspace_bytes, void *out, int32_t out_fp32, const int64_t *out_rows,
               int64_t ld_out, int32_t accumulate, void *stream);

/* Bytes of workspace tb_head_dh needs for these sizes on the current device (0 for no rows). No
 * counterpart in the reference. */
int64_t tb_head_dh_workspace(int64_t rows, int64_t cols, int64_t hidden_dim);

/* In place over the labelled rows of a [rows, cols] slab (columns col_offset ..):
 * logits <- fp16((exp(z - lse[row]) - [col == target]) * grad_scale); unlabelled rows untouched. */
int tb_head_dlogits(uint16_t *logits, const int64_t *targets, const float *lse, int64_t rows,
                    int64_t cols, int64_t ld, int64_t col_offset, float grad_scale, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TESTT_B200_H */
