/*
 * bdecode.h — C ABI of the B200 (sm_100a) decode-attention engine.
 *
 * Every entry point takes plain device pointers wrapped in `bd_tensor`
 * descriptors (data pointer, dtype code, shape and element strides — the same
 * information a DLPack DLTensor carries), a few scalars and a CUDA stream. No
 * entry point allocates device memory: scratch space comes from the caller as
 * (workspace, workspace_bytes), sized by the matching *_workspace() query, so
 * every launch is CUDA-graph capturable. Nothing synchronises the stream.
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

#ifdef __cplusplus
}
#endif
#endif /* BDECODE_H */
