/*
 * bdecode.h — C ABI of the B200 (sm_100a) decode-attention engine.
 *
 * Every entry point takes plain device pointers wrapped in `bd_tensor`
 * descriptors (data pointer, dtype code, shape and element strides — the same
 * information a DLPack DLTensor carries), a few scalars and a CUDA stream. No
 * entry point allocates device memory. Scratch space comes from the caller as
 * (workspace, workspace_bytes), sized by the matching *_workspace() query, so those
 * launches can be captured in CUDA graphs; bd_decode_attn_noalloc (below) instead
 * uses a fixed array inside the library. Nothing synchronises the stream.
 *
 * Return value: 0 (BD_OK) or a BD_ERR_* code; bd_last_error() gives the
 * message for the calling thread's last failure. Inputs are validated on the
 * host before any launch, so a rejected call launches nothing.
 *
 * Citations "ref: file:line" name the reference interface (saifmb0/bytes) the
 * entry point replaces; paths are relative to that project's root.
 */
#ifndef BDECODE_H
#define BDECODE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* bd_stream_t; /* identical to cudaStream_t */

enum bd_dtype {
  BD_F32 = 0, BD_F16 = 1, BD_BF16 = 2, BD_F8E4M3 = 3,
  BD_U8 = 4, BD_I8 = 5, BD_I32 = 6, BD_I64 = 7
};

enum bd_status {
  BD_OK = 0,
  BD_ERR_NULL = 1,        /* a required pointer or descriptor is NULL      */
  BD_ERR_DTYPE = 2,       /* unsupported or mismatched dtype               */
  BD_ERR_SHAPE = 3,       /* inconsistent or unsupported shape             */
  BD_ERR_STRIDE = 4,      /* layout the kernel cannot address              */
  BD_ERR_ALIGN = 5,       /* pointer / row pitch not 16-byte aligned       */
  BD_ERR_WORKSPACE = 6,   /* workspace missing or too small                */
  BD_ERR_UNSUPPORTED = 7, /* valid request this build does not implement   */
  BD_ERR_CUDA = 8,        /* CUDA runtime error (launch failure, etc.)     */
  BD_ERR_VALUE = 9        /* bad scalar argument (bits, k, group size ...) */
};

#define BD_MAX_DIMS 6
typedef struct bd_tensor {
  void* data;                   /* device pointer                     */
  int32_t dtype;                /* enum bd_dtype                      */
  int32_t ndim;                 /* <= BD_MAX_DIMS                     */
  int64_t shape[BD_MAX_DIMS];
  int64_t stride[BD_MAX_DIMS];  /* in elements                        */
} bd_tensor;

int bd_abi_version(void);
const char* bd_status_name(int status);
const char* bd_last_error(void);

/* Number of bounded device waits (TMA or bulk-copy barriers) on the current device that
 * ran past their iteration limit since the library was loaded; a non-zero count means
 * some earlier result is wrong. Synchronises the device (a diagnostic, not for the hot
 * path). Returns -1 if the counters cannot be read.
 * ref: none (the reference's Triton kernels have no bounded waits). */
long long bd_wait_timeouts(void);

/* ---------------------------------------------------------------------------
 * Dense GQA decode attention, split-KV (flash-decoding) with a log-sum-exp
 * combine. q [B,Hq,D] (the reference's [B,Hq,1,D] with the singleton dropped),
 * k,v [B,Hk,S,D] bf16 or fp8 e4m3 (same dtype), out [B,Hq,D] bf16/f16/f32.
 * scores = scaling * q.k (the reference wrappers apply no scale: pass 1.0).
 * ref: decode_attn_bf16  src/attention_kernels.py:65
 *      decode_attn_fp8   src/attention_kernels.py:156
 */
size_t bd_decode_attn_workspace(const bd_tensor* q, const bd_tensor* k);
int bd_decode_attn(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v,
                   const bd_tensor* out, float scaling, void* workspace,
                   size_t workspace_bytes, bd_stream_t stream);

/* bd_decode_attn without a caller workspace: no counterpart in the reference. For
 * callers that cannot allocate device memory for us (a serving runtime that reserves
 * all HBM for its KV pages at start-up, or a plain C / FFI host that only owns q, k, v
 * and out), the split partials go to a fixed 4 MiB device array inside the library,
 * which every GPU that loads the library keeps until the process exits. Calls needing
 * more split scratch than that are rejected with BD_ERR_UNSUPPORTED (use
 * bd_decode_attn then); nothing is allocated. Each call made outside a stream capture
 * looks up the array's device address on the current device (cudaGetSymbolAddress), so
 * a device reset never leaves a stale address; a call made while its stream is capturing
 * reuses the last address looked up, so make the first call on a device before any
 * stream capture.
 * All calls share the array, so calls that overlap on the GPU (other streams, other
 * host threads) race; serialise them. Every byte a call reads is written by that call. */
int bd_decode_attn_noalloc(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v,
                           const bd_tensor* out, float scaling, bd_stream_t stream);

/* Per-shard partials for split-KV across GPUs: m,l [B,Hq] f32 (running max of
 * scaling*q.k and softmax denominator), o [B,Hq,D] f32 (un-normalised
 * numerator). An empty shard yields m=-inf, l=0, o=0. Combine the shards of
 * all ranks with bd_lse_combine.
 * ref: no single counterpart — the reference is single-GPU; this is the shard
 *      step of decode_attn_bf16 (src/attention_kernels.py:33-61) cut at S/n. */
int bd_decode_attn_partial(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v,
                           float scaling, const bd_tensor* m, const bd_tensor* l,
                           const bd_tensor* o, void* workspace, size_t workspace_bytes,
                           bd_stream_t stream);

/* out[b,h] = sum_i o_i e^(m_i-M) / sum_i l_i e^(m_i-M), M = max_i m_i.
 * m,l [n,B,Hq] f32; o [n,B,Hq,D] f32; out [B,Hq,D] bf16/f16/f32. */
int bd_lse_combine(const bd_tensor* m, const bd_tensor* l, const bd_tensor* o,
                   const bd_tensor* out, bd_stream_t stream);

/* Split-KV across GPUs over NVLink peer memory. Each rank holds a contiguous token shard
 * k,v [B,Hk,S_r,D] of one sequence batch; every rank ends with the attention output over
 * all shards. `peer_buffers` is a DEVICE array of `world` pointers, entry r the base of
 * rank r's exchange buffer as this GPU addresses it (a symmetric allocation:
 * torch.distributed._symmetric_memory, or cuMem handles mapped on every GPU), each
 * bd_peer_exchange_buffer_bytes(B*Hq, D, world) bytes and zeroed once before the first call
 * (it holds the per-row step counters, so it must not be cleared between steps). Every rank
 * calls with the same shapes, one call per step, on one stream; calls may be captured in a
 * CUDA graph and replayed. One kernel (at most one CTA per SM, each over rows b*Hq + hq)
 * merges this rank's split partials per row, stores the merged (max, sum, numerator) into
 * every rank's buffer, raises a per-step flag on each, waits (at most 1 s; then the rows of
 * that CTA are NaN and bd_wait_timeouts() counts it) for all ranks' flags and writes the
 * log-sum-exp combine.
 *   bd_split_kv_decode_peer: the whole step -- the dense split pass over this rank's shard
 *     (q [B,Hq,D], k,v bf16 or fp8 e4m3 as bd_decode_attn; workspace of
 *     bd_decode_attn_workspace(q, k) bytes) and the exchange kernel, launched as its
 *     programmatic dependent (two launches, no separate merge kernel).
 *   bd_peer_exchange_combine: the exchange of partials the caller computed (m, l [B,Hq],
 *     o [B,Hq,D] f32, as bd_decode_attn_partial returns them).
 * out [B,Hq,D] bf16/f16/f32. Needs D a multiple of 4, at most 512; world <= 64.
 * ref: no single counterpart -- the reference is single-GPU; this is split-KV decode across
 *      GPUs (the merge identity of src/attention_kernels.py:45-59 applied to shards). */
size_t bd_peer_exchange_buffer_bytes(int rows, int D, int world);
int bd_split_kv_decode_peer(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, float scaling,
                            void* const* peer_buffers, int rank, int world, const bd_tensor* out,
                            void* workspace, size_t workspace_bytes, bd_stream_t stream);
int bd_peer_exchange_combine(const bd_tensor* m, const bd_tensor* l, const bd_tensor* o,
                             void* const* peer_buffers, int rank, int world, const bd_tensor* out,
                             bd_stream_t stream);

/* ---------------------------------------------------------------------------
 * KIVI 2/4-bit KV-cache decode: a packed-cache split-KV kernel, then a bf16
 * residual-window kernel that (when the window takes one CTA per head group) also
 * merges the split partials into `out`; otherwise a log-sum-exp combine follows.
 * Q [B,Hq,D=128] bf16/f16/f32;
 * Kq int32 [B,Hk,D,Sq*bits/32]; K_scale,K_mn f16 [B,Hk,D,Sq/32];
 * Vq int32 [B,Hk,Sq,D*bits/32]; V_scale,V_mn f16 [B,Hk,Sq,D/32];
 * K_residual,V_residual bf16 [B,Hk,R,D]; out [B,Hq,D]; group_size 32.
 * scaling multiplies q.k (the reference step uses 1/sqrt(D)).
 * Row pitches: Kq/Vq rows 16-byte aligned, scale/min rows 8-byte aligned.
 * ref: kivi_decode_attn  benchmarks/kivi_latency.py:59 (which calls the external
 *      cuda_bmm_fA_qB_outer twice plus torch matmul/softmax) */
size_t bd_kivi_decode_attn_workspace(const bd_tensor* Q, const bd_tensor* Kq, const bd_tensor* K_residual,
                                     int bits);
int bd_kivi_decode_attn(const bd_tensor* Q, const bd_tensor* Kq, const bd_tensor* K_scale, const bd_tensor* K_mn,
                        const bd_tensor* K_residual, const bd_tensor* Vq, const bd_tensor* V_scale,
                        const bd_tensor* V_mn, const bd_tensor* V_residual, int bits, int group_size, float scaling,
                        const bd_tensor* out, void* workspace, size_t workspace_bytes, bd_stream_t stream);

/* Profiling form of bd_kivi_decode_attn: launches only the selected stages of the
 * step (bit 0: packed-cache split kernel, bit 1: residual-window kernel, bit 2:
 * merge into `out`). stages = 7 is bd_kivi_decode_attn. Used to time kernels one by one.
 * ref: none (measurement helper around kivi_decode_attn). */
int bd_kivi_decode_attn_stages(const bd_tensor* Q, const bd_tensor* Kq, const bd_tensor* K_scale,
                               const bd_tensor* K_mn, const bd_tensor* K_residual, const bd_tensor* Vq,
                               const bd_tensor* V_scale, const bd_tensor* V_mn, const bd_tensor* V_residual, int bits,
                               int group_size, float scaling, const bd_tensor* out, void* workspace,
                               size_t workspace_bytes, int stages, bd_stream_t stream);

/* Group-wise asymmetric quantize + pack along the last dim: per group of 32,
 * scale = max(max-min, 1e-8)/(2^bits-1) (fp32, IEEE divide), code =
 * clamp(round_half_even((x-min)/scale)); element e -> word e/(32/bits), bit
 * offset (e%(32/bits))*bits. x [...,N] f16/bf16/f32 (1-4 dims); code int32
 * [...,N*bits/32]; scale, mn [...,N/32] in x's dtype (all contiguous).
 * ref: triton_quantize_and_pack_along_last_dim (external KIVI, called at
 *      benchmarks/kivi_latency.py:123; layout pinned by :26-35) */
int bd_kivi_pack_last_dim(const bd_tensor* x, int group_size, int bits, const bd_tensor* code,
                          const bd_tensor* scale, const bd_tensor* mn, bd_stream_t stream);

/* Streaming KIVI cache write: quantizes whole 32-token groups of new keys and values
 * into existing packed caches, starting at token `token_offset` (a multiple of 32).
 * Keys go per channel over each group's tokens, values per token over 32-channel
 * groups, with bd_kivi_pack_last_dim's arithmetic, so after any sequence of appends the
 * caches equal packing the whole sequence at once. k_new, v_new [B,Hk,Tn,D]
 * f16/bf16/f32 (Tn, D multiples of 32, channels contiguous); Kq int32 [B,Hk,D,>=end/fpi],
 * K_scale/K_mn f16 [B,Hk,D,>=end/32], Vq int32 [B,Hk,>=end,D/fpi], V_scale/V_mn f16
 * [B,Hk,>=end,D/32] with end = token_offset + Tn (fpi = 32/bits); cache rows contiguous,
 * other strides free. This is the step before the decode path: a serving loop flushes
 * the oldest 32 tokens of the bf16 residual window once it exceeds R.
 * ref: the reference packs whole tensors (external KIVI packer, benchmarks/kivi_latency.py:123)
 *      and keeps the newest R tokens exact (KIVIQuantizer, src/quantization.py:468-501);
 *      it has no incremental append. */
int bd_kivi_append(const bd_tensor* k_new, const bd_tensor* v_new, int bits, int group_size, int64_t token_offset,
                   const bd_tensor* Kq, const bd_tensor* K_scale, const bd_tensor* K_mn, const bd_tensor* Vq,
                   const bd_tensor* V_scale, const bd_tensor* V_mn, bd_stream_t stream);

/* out[b,hq,m,n] = sum_k fA[b,hq,m,k] * (code(qB)[b,hq/G,k,n]*scales + zeros), f16.
 * fA f16 [B,Hq,M,K]; qB int32 [B,Hk,K,N*bits/32]; scales,zeros f16
 * [B,Hk,K,N/group_size]; out f16 [B,Hq,M,N].
 * ref: cuda_bmm_fA_qB_outer (external KIVI, called at benchmarks/kivi_latency.py:67,83) */
int bd_kivi_gemv_outer(int group_size, const bd_tensor* fA, const bd_tensor* qB, const bd_tensor* scales,
                       const bd_tensor* zeros, int bits, const bd_tensor* out, bd_stream_t stream);

/* ---------------------------------------------------------------------------
 * Pass-1 scores [B,Hq,S] f32 = scaling * q.k over all keys.
 * score_bits 16: k bf16, f16 or f32 [B,Hk,S,D];  8: k fp8 e4m3 [B,Hk,S,D];
 * 4 / 2: k uint8 [B,Hk,S,D*bits/8] (channel c at byte c/(8/bits), shift
 * (c%(8/bits))*bits), key = code*scale + zero with scale/zero bf16 or f16
 * [B,Hk,S,D/group_size] (token-major, contiguous per (b,h)). q bf16/f16/f32.
 * A bf16 query over bf16 keys, or a bf16/f16 query over fp8 or packed keys, runs on
 * the tensor cores (products exact in fp32); an fp32 query, an f16 query over bf16
 * keys, f16/f32 keys and head_dim 32 run in fp32 on the CUDA cores, unrounded.
 * head_dim 32, 64 or 128.
 * ref: sparse_score_scalar  src/attention_kernels.py:1113
 *      sparse_score_packed  src/attention_kernels.py:1199 */
int bd_sparse_score(const bd_tensor* q, const bd_tensor* k, const bd_tensor* scale, const bd_tensor* zero,
                    float scaling, int score_bits, int group_size, const bd_tensor* scores, bd_stream_t stream);

/* Per-token groups of group_size channels: fp32 min/max, scale =
 * max(max-min,1e-8)/(2^bits-1), code = clamp(round_half_even((k-min)/scale)),
 * 8/bits codes per byte, low bits first. k [B,H,S,D] bf16/f16/f32; packed u8
 * [B,H,S,D*bits/8]; scale, zero (= min) [B,H,S,D/group_size] in k's dtype.
 * ref: quantize_and_pack_score_keys  src/attention_kernels.py:1225 */
int bd_pack_score_keys(const bd_tensor* k, int score_bits, int group_size, const bd_tensor* packed,
                       const bd_tensor* scale, const bd_tensor* zero, bd_stream_t stream);

/* Top-k along the last dim of scores [R] / [R0,R1] / [B,R1,n] f32: keys larger
 * first, equal values keep the lower index first (a stable descending sort).
 * sorted=1 orders the k winners by (value desc, index asc); sorted=0 returns
 * them in ascending index order. values (optional) f32 and indices int64/int32
 * have k in the last dim. k <= n.
 * ref: scores.topk(kb, dim=-1)  src/attention_kernels.py:1069,1262
 *      select_topk('exact')     benchmarks/sparse_attention.py:287-309 */
int bd_topk(const bd_tensor* scores, int k, int sorted, const bd_tensor* values, const bd_tensor* indices,
            bd_stream_t stream);

/* Exact softmax(scaling * q.k_sel) . v_sel over per-query-head key positions
 * idx [B,Hq,kb] (int32/int64; duplicates count once per occurrence, positions
 * outside [0,S) are skipped). q [B,Hq,D] bf16/f16/f32; k,v [B,Hk,S,D] of one
 * dtype: bf16, fp8 e4m3, f16 or f32 (widened to fp32); out [B,Hq,D] bf16/f16/f32
 * (bf16 for fp8 values in the reference).
 * ref: sparse_gather_attn  src/attention_kernels.py:1037; attend_topk
 *      benchmarks/sparse_attention.py:367 */
size_t bd_sparse_gather_attn_workspace(const bd_tensor* q, const bd_tensor* idx);
int bd_sparse_gather_attn(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, const bd_tensor* idx,
                          float scaling, const bd_tensor* out, void* workspace, size_t workspace_bytes,
                          bd_stream_t stream);

/* Shard step of a sparse decode whose keys are split across GPUs: the same gather-attend
 * over this device's selected positions (others -1 or out of range), exported as one
 * (m, l, o) per (b, q-head) for bd_lse_combine after an all-gather -- m,l [B,Hq] f32
 * (m in natural-log units of scaling*q.k), o [B,Hq,D] f32 un-normalised, all contiguous.
 * Same workspace as bd_sparse_gather_attn.
 * ref: no single counterpart -- the reference is single-GPU; this is attend_topk
 *      (benchmarks/sparse_attention.py:367) cut at a shard of the positions. */
int bd_sparse_gather_attn_partial(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v,
                                  const bd_tensor* idx, float scaling, const bd_tensor* m, const bd_tensor* l,
                                  const bd_tensor* o, void* workspace, size_t workspace_bytes,
                                  bd_stream_t stream);

/* Quest page metadata: elementwise min / max of each page of `page` tokens
 * (a ragged last page covers the real tokens only). k [B,H,S,D]; kmin, kmax
 * [B,H,ceil(S/page),D] in k's dtype, channels contiguous, other strides free -- so a
 * serving loop refreshes pages [p0, p1) of a metadata cache by passing the views
 * k[:, :, p0*page : min(S, p1*page)] and kmin/kmax[:, :, p0:p1].
 * ref: _quest_select  benchmarks/sparse_attention.py:334-341 */
int bd_quest_page_minmax(const bd_tensor* k, int page, const bd_tensor* kmin, const bd_tensor* kmax,
                         bd_stream_t stream);
/* bound[b,hq,p] = scaling * sum_d max(q_d*kmin_pd, q_d*kmax_pd) (fp32), with
 * pages p >= force_from_page set to +inf (the reference's forced recent window;
 * pass a value >= np for none). kmin/kmax [B,Hk,np,D] bf16, f16 or f32 (both one
 * dtype, read unrounded); q bf16/f16/f32; bounds f32 [B,Hq,np].
 * ref: benchmarks/sparse_attention.py:342-355 */
int bd_quest_page_bounds(const bd_tensor* q, const bd_tensor* kmin, const bd_tensor* kmax, float scaling,
                         int force_from_page, const bd_tensor* bounds, bd_stream_t stream);
/* Page bounds -> top npick = min(max(1,ceil(kb/page)), np) pages (lower page
 * wins ties, ordered by bound desc) -> token indices page*p + o clamped to S-1:
 * idx [B,Hq,npick*page] int32/int64.
 * ref: _quest_select  benchmarks/sparse_attention.py:356-364 */
size_t bd_quest_select_workspace(const bd_tensor* q, const bd_tensor* kmin, int kb, int page);
int bd_quest_select(const bd_tensor* q, const bd_tensor* kmin, const bd_tensor* kmax, int S, int kb, int page,
                    float scaling, int force_from_page, const bd_tensor* idx_out, void* workspace,
                    size_t workspace_bytes, bd_stream_t stream);

/* ---------------------------------------------------------------------------
 * PQ-LUT decode: scores[t] = sum_j lut[b,hq,j,k_idx[t,j]] (+ sum_c q_out[hq,c] *
 * k_out[t,c] when k_out is given, C_out <= 8), softmax, then P.V with V one of:
 * bf16 / fp8 e4m3 [.,Hk,S,D] (v), int8 [B,Hk,S,D] with f16 per-token v_scale
 * [B,Hk,S], or PQ codes v_idx u8 [.,Hk,S,M_v] + v_centroids f32 [M_v,K_v,d_sub_v].
 * Paged when block_table int32 [B,max_blocks] and context_lens int32 [B] are
 * given (k_idx / k_out / values then [num_blocks,Hk,block_size,.]).
 * lut f32 [B,Hq,M,K] (M <= 64, K <= 256); k_idx u8; out [B,Hq,D].
 * ref: decode_attn_pq_lut        src/attention_kernels.py:365
 *      decode_attn_pq_lut_kv     src/attention_kernels.py:471
 *      paged_attn_pq_lut_kv      src/attention_kernels.py:588
 *      decode_attn_pq_lut_asym   src/attention_kernels.py:713
 *      paged_attn_pq_lut_asym    src/attention_kernels.py:858
 *      (int8 values: configuration extension, no counterpart in the reference) */
size_t bd_pq_decode_workspace(const bd_tensor* lut, const bd_tensor* k_idx, const bd_tensor* v,
                              const bd_tensor* v_idx, const bd_tensor* v_centroids, const bd_tensor* block_table,
                              const bd_tensor* context_lens, int block_size);
int bd_pq_decode(const bd_tensor* lut, const bd_tensor* k_idx, const bd_tensor* k_out, const bd_tensor* q_out,
                 const bd_tensor* v, const bd_tensor* v_scale, const bd_tensor* v_idx, const bd_tensor* v_centroids,
                 const bd_tensor* block_table, const bd_tensor* context_lens, int block_size, const bd_tensor* out,
                 void* workspace, size_t workspace_bytes, bd_stream_t stream);
/* Scores only [B,Hq,S] f32 (LUT + outliers).
 * ref: sparse_score_pq_lut_asym  src/attention_kernels.py:960 */
int bd_pq_scores(const bd_tensor* lut, const bd_tensor* k_idx, const bd_tensor* k_out, const bd_tensor* q_out,
                 const bd_tensor* scores, bd_stream_t stream);
/* lut[b,h,j,c] = sum_i q[b,h,j*d_sub+i] * centroids[j,c,i]; q [B,H,D]; centroids f32
 * [M,K,d_sub]; lut f32 [B,H,M,K] contiguous.
 * ref: the LUT einsum of benchmarks/test_correctness.py:181-182 and the key
 *      reconstruction of decode_attn_dequant src/attention_kernels.py:267 */
int bd_pq_build_lut(const bd_tensor* q, const bd_tensor* centroids, const bd_tensor* lut, bd_stream_t stream);
/* codes[n,j] = argmax_c (x_h . c_h - norm_c), first index on ties: the reference's CUDA
 * nearest-centroid rule (x and the centroids rounded to f16 -- the centroids through x's
 * dtype first -- products summed in fp32, norm_c = 0.5*||c||^2 rounded to x's dtype).
 * x [N,D] f32/bf16/f16; codes [N,M] u8 or int64. For d_sub > 16 the whole sub-vector is
 * used (the reference's CUDA kernel reads its first 16 elements only).
 * ref: ProductQuantizer.quantize  src/quantization.py:160-199 (CUDA branch) */
int bd_pq_encode(const bd_tensor* x, const bd_tensor* centroids, const bd_tensor* codes, bd_stream_t stream);

/* Asymmetric uniform fake-quant over axis 3 of a 5-d strided view x (o0,o1,o2,
 * group,inner): y = clamp(round((x-min)/scale),0,levels-1)*scale + min with scale =
 * clamp(max-min,1e-8)/(levels-1), every step rounded in x's dtype (f32/bf16/f16);
 * y contiguous, same shape and dtype.
 * ref: _asym_uniform_fakequant  src/quantization.py:432; KIVIQuantizer
 *      quantize_key / quantize_value  src/quantization.py:468-501 */
int bd_asym_fakequant(const bd_tensor* x, int levels, const bd_tensor* y, bd_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* BDECODE_H */
