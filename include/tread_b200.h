/*
 * tread_b200 C ABI: B200 (sm_100a) kernels for tread's chunk-reuse hot path.
 *
 * The reference (sykeriin/tread) is pure Python/PyTorch and has no FFI; each entry point
 * below replaces the library-call sequence at the cited reference location, and the
 * Python host layer (package `tread_b200`) keeps tread's own function signatures on top.
 *
 * Conventions for every entry point:
 *   - returns TREAD_OK (0) or a nonzero status; tread_last_error() then describes it;
 *   - tensor pointers are DEVICE pointers owned by the caller (PyTorch); arrays documented
 *     as "host" are read during the call only;
 *   - all work is stream-ordered on `stream` (a cudaStream_t); no call synchronises the
 *     host, and none allocates device memory unless its comment says so;
 *   - no C++ exception crosses the boundary.
 */
#ifndef TREAD_B200_H
#define TREAD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* tread_stream_t; /* identical to cudaStream_t */

enum {
  TREAD_OK = 0,
  TREAD_ERR_INVALID = 1, /* bad argument: nothing was launched */
  TREAD_ERR_CUDA = 2,    /* CUDA runtime error at launch */
  TREAD_ERR_TIMEOUT = 3  /* a bounded device-side wait gave up */
};

/* element type codes for the `dtype` arguments */
enum { TREAD_F32 = 0, TREAD_F16 = 1, TREAD_BF16 = 2 };

/* Text of the last error raised on the calling host thread ("" if none). */
const char* tread_last_error(void);

/* ABI revision of this library; bumped on any signature change, new entry point or newly accepted flag
 * (4: tread_attn_rows accepts TREAD_ATTN_FORCE_TAIL_SPLIT; 5: tread_rows_gemm). */
int tread_abi_version(void);

/*
 * Fused gather + RoPE re-rotation + append of cached KV blocks into one assembled cache.
 *
 * Replaces, per request, the loop at tread/engine.py:108-120:
 *   Ks.append(rotate_keys(model, b.K, offset - b.base)); Vs.append(b.V)   (engine.py:112-115)
 *   K = torch.cat(Ks, dim=-2); V = torch.cat(Vs, dim=-2)                  (engine.py:119-120)
 * with rotate_keys (tread/blend.py:22-39) computed in fp32:
 *   angle_i = float(delta) * inv_freq[i]       (fp32 product, as HF rotary_emb)
 *   c_i = cos(angle_i) * s / s,  s_i = sin(angle_i) * s / s   (s = attention_scaling)
 *   out[i]       = x[i] * c_i - x[i + D/2] * s_i
 *   out[i + D/2] = x[i + D/2] * c_i + x[i] * s_i          (rotate_half pairing)
 * rounded once to the storage type. delta == 0 copies K unchanged (blend.py:32-33).
 *
 * Segment j (0 <= j < nseg) is one cached block, K and V each laid out contiguous as
 * [L, Hkv, n_tok[j], D] (tread/store.py:1-5 layout, batch dim of 1 dropped). Its tokens
 * land at token rows dst_tok0[j] .. dst_tok0[j] + n_tok[j] - 1 of out_k / out_v, which
 * are [L, Hkv, T_out, D] contiguous. Segments must not overlap in the output.
 *
 *   k_src, v_src : host arrays [nseg] of device pointers (16-byte aligned)
 *   n_tok        : host [nseg], each >= 0
 *   delta        : host [nseg] position shift (new offset - base), |delta| < 2^24
 *   dst_tok0     : host [nseg]
 *   inv_freq     : host [D/2] fp32 RoPE inverse frequencies (model.rotary_emb.inv_freq)
 *   attn_scaling : RoPE attention scaling folded into HF cos/sin (1.0 for default RoPE)
 *   dtype        : TREAD_BF16, TREAD_F16 or TREAD_F32; D * elsize a multiple of 32 bytes
 */
int tread_rope_gather_append(const void* const* k_src, const void* const* v_src,
                             const int32_t* n_tok, const int64_t* delta,
                             const int64_t* dst_tok0, int nseg, void* out_k, void* out_v,
                             int L, int Hkv, int D, int64_t T_out, const float* inv_freq,
                             float attn_scaling, int dtype, tread_stream_t stream);

/*
 * Fused layer-1 KV deviation + top-k selection (CacheBlend-style token selector).
 *
 * Replaces tread/blend.py:129 (per-candidate deviation), :160 (dev.topk(budget)) and :165
 * (S.sort()) in one launch:
 *   dev[t] = sum_h ||k1[h,t] - K1[h,pos_t]||_2 + sum_h ||v1[h,t] - V1[h,pos_t]||_2
 * in fp32 with a fixed summation order (per head: 32 lanes of D/32 consecutive elements
 * accumulated in order, xor-butterfly 16,8,4,2,1, IEEE sqrt; heads summed in order; K sum
 * plus V sum), then the `budget` largest dev values (ties -> lower candidate index) written
 * as ascending candidate indices to sel_idx and their positions cand_pos[sel_idx] to sel_pos.
 *
 *   k1, v1     : fresh layer-1 rows; element (h, t, d) at t*fresh_stride_tok +
 *                h*fresh_stride_head + d (elements)
 *   K1, V1     : layer-1 assembled cache; element (h, p, d) at p*cache_stride_tok +
 *                h*cache_stride_head + d; positions must lie in [0, T_cache)
 *   cand_pos   : device int64 [n], candidate positions (tread's all_c)
 *   D          : 64, 128 or 256; rows aligned to D/32 elements
 *   dev_out    : device fp32 [n]; sel_idx, sel_pos : device int64 [budget] (sel_pos may be NULL)
 *   workspace  : device buffer of TREAD_DEVIATION_WORKSPACE_BYTES, zero-filled once by the
 *                caller; word 0 is a CTA ticket the kernel returns to zero, word 1 a sticky
 *                flag set to 1 if a candidate position was out of range (that dev is NaN).
 *                Calls sharing a workspace must be stream-ordered.
 */
#define TREAD_DEVIATION_WORKSPACE_BYTES 256
int tread_deviation_topk(const void* k1, const void* v1, int64_t fresh_stride_tok,
                         int64_t fresh_stride_head, const void* K1, const void* V1,
                         int64_t cache_stride_tok, int64_t cache_stride_head, int64_t T_cache,
                         const int64_t* cand_pos, int n, int Hkv, int D, int budget, int dtype,
                         float* dev_out, int64_t* sel_idx, int64_t* sel_pos, void* workspace,
                         tread_stream_t stream);

/*
 * The same selector split for KV-head tensor parallelism (the reference is single-GPU; this
 * is tread/blend.py:129,160,165 with the head sum spread over ranks). Each rank holds the
 * contiguous head slice [r*Hkv, (r+1)*Hkv) of the layer-1 rows and cache:
 *
 * tread_deviation_head_norms writes norms_out, device fp32 [2][Hkv][n]:
 *   norms_out[0][h][t] = ||k1[h,t] - K1[h,pos_t]||_2,  norms_out[1][h][t] = same for v1/V1,
 * each computed exactly as inside tread_deviation_topk (same element/lane/butterfly order).
 * Arguments as for tread_deviation_topk (Hkv <= 32); workspace word 1 is the same sticky
 * out-of-range flag (those norms are NaN).
 *
 * tread_select_head_norms takes the all-gathered norms of every head, device fp32 [2][H][n]
 * in global head order, forms dev[t] = (((nk_0 + nk_1) + ...) + ((nv_0 + nv_1) + ...)) -- the
 * fused kernel's order, so the result equals a single-GPU tread_deviation_topk bit for bit --
 * and selects exactly as tread_deviation_topk does (dev_out, sel_idx, sel_pos, workspace alike).
 */
int tread_deviation_head_norms(const void* k1, const void* v1, int64_t fresh_stride_tok,
                               int64_t fresh_stride_head, const void* K1, const void* V1,
                               int64_t cache_stride_tok, int64_t cache_stride_head, int64_t T_cache,
                               const int64_t* cand_pos, int n, int Hkv, int D, int dtype,
                               float* norms_out, void* workspace, tread_stream_t stream);
int tread_select_head_norms(const float* norms, int n, int Hkv, int budget, const int64_t* cand_pos,
                            float* dev_out, int64_t* sel_idx, int64_t* sel_pos, void* workspace,
                            tread_stream_t stream);

/*
 * Allocation-free variant of tread_deviation_topk. It has no counterpart in the reference; it
 * exists for callers that cannot provide device scratch: serving loops whose device memory is
 * owned by a pooling allocator reserved at start-up, loops that avoid cudaMalloc because it can
 * synchronise the device, and FFI hosts with no device allocator. The selector's scratch (ticket
 * and error words plus the fp32 deviation of every candidate) lives in a file-scope device array
 * of 256 B + 4 B x TREAD_NOALLOC_MAX_CANDIDATES (about 256 KB) that every GPU loading the
 * library holds until exit; the caller passes the same inputs and the sel_idx / sel_pos outputs
 * as for tread_deviation_topk (the deviation values themselves are not returned).
 *   - n > TREAD_NOALLOC_MAX_CANDIDATES is rejected with TREAD_ERR_INVALID;
 *   - every call looks up the array's device address in the current context
 *     (cudaGetSymbolAddress), so it stays right after cudaDeviceReset; make the first call on a
 *     device before any stream capture (it loads the module);
 *   - every call clears the ticket words on `stream` and then reuses the shared array, so calls
 *     that overlap on the GPU (different streams, or different host threads) race: order them;
 *   - err_flag (optional, device unsigned[1], may be NULL) receives this call's out-of-range
 *     flag in stream order: 1 if a candidate position lay outside [0, T_cache) (that candidate's
 *     deviation is NaN and it ranks first), else 0. It is copied out of the shared array, so it
 *     needs no scratch from the caller;
 *   - it calls no cudaMalloc / cudaFree.
 */
#define TREAD_NOALLOC_MAX_CANDIDATES 65536
int tread_deviation_topk_noalloc(const void* k1, const void* v1, int64_t fresh_stride_tok,
                                 int64_t fresh_stride_head, const void* K1, const void* V1,
                                 int64_t cache_stride_tok, int64_t cache_stride_head, int64_t T_cache,
                                 const int64_t* cand_pos, int n, int Hkv, int D, int budget, int dtype,
                                 int64_t* sel_idx, int64_t* sel_pos, unsigned* err_flag,
                                 tread_stream_t stream);

/*
 * RoPE at each row's absolute position + splice of the row's K/V into the layer cache.
 *
 * Replaces, per recomputed layer, tread/blend.py:82-90 (`_qkv`: q/k/v views of the
 * projections and apply_rotary_pos_emb at positions S) and tread/blend.py:106
 * (`K[:, :, S], V[:, :, S] = k, v`). Row r of `qkv` ([R, ld_qkv], columns [q heads | k heads
 * | v heads] of D each) sits at position pos[r]:
 *   q_out[r, h, :]            = rope(q_h, pos[r])          (q_out: [R, Hq, D] contiguous)
 *   K_cache[g*cs + pos[r]*D]  = rope(k_g, pos[r]);  V_cache[...] = v_g
 * with cos/sin(float(pos) * inv_freq[i]) * attn_scaling in fp32, rounded once to `dtype`.
 * The caches are one layer's [Hkv, T_cache, D] with head stride cache_stride_head (elements).
 * A position outside [0, T_cache) skips its row and sets bit 0 of *err_flag (may be NULL).
 * kv_by_row = 1 writes row r's k/v to cache row r instead of row pos[r] (dense [Hkv, R, D]
 * outputs, e.g. the fresh layer-1 rows of the deviation selector, blend.py:128); q_out may be
 * NULL to skip the q heads. With q_out NULL, Hq = 0 declares rows of [k heads | v heads] only
 * (a k/v-only projection: the selector needs no layer-1 queries, blend.py:127-129).
 */
int tread_rope_rows(const void* qkv, int64_t ld_qkv, const int64_t* pos, int R, int Hq, int Hkv, int D,
                    void* q_out, void* K_cache, void* V_cache, int64_t cache_stride_head,
                    int64_t T_cache, int kv_by_row, const float* inv_freq, float attn_scaling,
                    int dtype, void* err_flag, tread_stream_t stream);

/*
 * Recompute attention: each row attends, per query head, to every cache key at a position
 * <= its own, with GQA (query head h reads KV head h / (Hq/Hkv)).
 *
 * Replaces tread/blend.py:76 (mask[s, t] = t <= S[s]) and tread/blend.py:110
 * (F.scaled_dot_product_attention(q, repeat_kv(K, g), repeat_kv(V, g), attn_mask=mask)),
 * and, with the query segment's rows appended, the query forward's attention
 * (tread/engine.py:131-132). q, out: [R, Hq, D]; K/V: one layer's [Hkv, T_cache, D] at head
 * stride cache_stride_head; softmax in fp32 with scores scaled by sm_scale. Positions outside
 * [0, T_cache) skip their row and set bit 1 of *err_flag (may be NULL).
 * bf16 / fp16 with D == 128 run on the tcgen05 tensor-core kernel (TMA-fed, S, P and O in
 * TMEM). A bounded mbarrier wait that gives up sets bit 2 of *err_flag. flags bit 0 forces the
 * CUDA-core kernel (used for fp32 and the other head dims); bit 1 selects the stream-K schedule and
 * bit 2 the tail-split schedule explicitly (bits 1 and 2 together are rejected).
 *
 * workspace (device, 256-byte aligned, tread_attn_rows_workspace_bytes() of it, zero-filled once by
 * the caller; may be NULL): with it, the tensor-core kernel runs one CTA per SM over whole 128-row
 * tiles, longest first, and splits the tiles left after the last full round into key ranges over
 * the CTAs (tail split; stream-K instead gives every CTA an equal share of all tiles' key blocks).
 * Tiles split between CTAs are merged from partial results kept in the workspace; the kernel
 * returns its counters to zero, except after an error of bit 2, when the caller must zero the
 * workspace again. Without it each CTA runs one whole tile. Calls that share a workspace must be
 * stream-ordered.
 */
#define TREAD_ATTN_FORCE_CUDA_CORES 1
#define TREAD_ATTN_FORCE_STREAM_K 2
#define TREAD_ATTN_FORCE_TAIL_SPLIT 4
size_t tread_attn_rows_workspace_bytes(void);
int tread_attn_rows(const void* q, const void* K_cache, const void* V_cache, int64_t cache_stride_head,
                    int64_t T_cache, const int64_t* q_pos, int R, int Hq, int Hkv, int D, float sm_scale,
                    void* out, int dtype, int flags, void* err_flag, void* workspace,
                    size_t workspace_bytes, tread_stream_t stream);

/*
 * Fused RMSNorm over rows: y[r] = to_dtype(w * to_dtype(x[r] * rsqrt(mean(x[r]^2) + eps))), fp32
 * inside. Replaces the HF Qwen2RMSNorm calls on the recomputed rows (tread/blend.py:105,113 via
 * layer.input_layernorm / post_attention_layernorm), one pass instead of ~8 kernels.
 * x, y: [rows, hidden] at row strides ld_x / ld_y (elements); weight [hidden]; 16-byte aligned.
 */
int tread_rmsnorm(const void* x, int64_t ld_x, const void* weight, void* y, int64_t ld_y, int64_t rows,
                  int hidden, float eps, int dtype, tread_stream_t stream);

/*
 * Fused SwiGLU activation: y[r, i] = to_dtype(to_dtype(silu(g[r, i])) * u[r, i]) with
 * gate_up[r] = [g | u] (2 * inter columns). Replaces act_fn(gate_proj(x)) * up_proj(x) of HF
 * Qwen2MLP on the recomputed rows (tread/blend.py:113), one pass instead of two kernels.
 */
int tread_silu_mul(const void* gate_up, int64_t ld_gu, void* y, int64_t ld_y, int64_t rows, int inter,
                   int dtype, tread_stream_t stream);

/*
 * Few-row projection GEMM on the tensor cores:
 *   out[M, N] = (accumulate ? out : 0) + x[M, K] w[N, K]^T + bias[N]
 * fp32 accumulation, rounded once to dtype. It replaces the Linear layers of the query forward when
 * only the query segment's rows run (tread/engine.py:131-132: the q/k/v, o_proj, gate/up, down
 * projections and lm_head of model(query_ids, past_key_values=cache)); there the weights dominate
 * the traffic and the GEMM is bound by HBM. 1 <= M <= 128.
 * bf16 / fp16 only. x, w, out: row-major at row strides ldx, ldw, ld_out (elements). x and w must be
 * 16-byte aligned, and K, ldx and ldw multiples of 8. bias (length N) may be NULL. out must not
 * overlap x or w.
 * workspace: NULL, or tread_rows_gemm_workspace_bytes() of device memory, 256-byte aligned (its
 * contents on entry do not matter). With it, weights with fewer 256-feature pairs than SMs are split
 * along K over more CTAs, and a second launch adds the splits' partial sums in split order, so the
 * result does not depend on timing. Calls that share a workspace must be stream-ordered. A bounded
 * wait that gives up sets bit 2 of *err_flag (may be NULL).
 */
size_t tread_rows_gemm_workspace_bytes(void);
int tread_rows_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias, void* out,
                    int64_t ld_out, int M, int N, int K, int accumulate, int dtype, void* err_flag,
                    void* workspace, size_t workspace_bytes, tread_stream_t stream);

/*
 * Block-store tier transfers (pinned host <-> HBM), stream-ordered DMA copies.
 *
 * tread_kv_spill replaces the GPU->CPU-tier move of tread/store.py:111
 * (`b.K.to("cpu").pin_memory()`: a synchronous pageable copy plus a second pinned copy) and
 * tread_kv_fetch the CPU-tier hit of tread/store.py:75-76 (`b.K.to(b.device,
 * non_blocking=True)`). Issue them on a transfer stream and order consumers with events so
 * the copies overlap rotation kernels on the compute stream.
 * Host buffers must be page-locked (cudaHostAlloc / torch pin_memory); TREAD_ERR_INVALID
 * otherwise. The *_rows variants copy `nrows` rows of `row_bytes` at the given pitches
 * (one block's token slice of an assembled [L, Hkv, T, D] cache is L*Hkv such rows).
 */
int tread_kv_fetch(void* dst_device, const void* src_host, size_t bytes, tread_stream_t stream);
int tread_kv_spill(void* dst_host, const void* src_device, size_t bytes, tread_stream_t stream);
int tread_kv_fetch_rows(void* dst_device, size_t dst_pitch, const void* src_host, size_t src_pitch,
                        size_t row_bytes, size_t nrows, tread_stream_t stream);
int tread_kv_spill_rows(void* dst_host, size_t dst_pitch, const void* src_device, size_t src_pitch,
                        size_t row_bytes, size_t nrows, tread_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* TREAD_B200_H */
