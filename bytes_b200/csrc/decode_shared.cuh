// Pieces shared by the split-KV decode kernels: partial-result layout and the
// launcher of the dense bf16/fp8 split kernel used for residual windows.
#pragma once
#include "common.cuh"

namespace bd {

// Split partials live in a float workspace: m[rows*nsplit], l[rows*nsplit],
// o[rows*nsplit*D], rows = B*Hq, partial index (b*Hq + hq)*nsplit + split.
struct Partials {
  float* m; float* l; float* o;
  int nsplit;  // total splits in the buffer (stride)
};

// o first, so every partial row of D floats starts on a 16-byte boundary when D % 4 == 0
inline Partials carve_partials(void* ws, size_t rows, int nsplit, int D) {
  float* base = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
  Partials p;
  p.o = base;
  p.m = base + rows * nsplit * size_t(D);
  p.l = p.m + rows * nsplit;
  p.nsplit = nsplit;
  return p;
}
inline size_t partials_bytes(size_t rows, int nsplit, int D) {
  return rows * size_t(nsplit) * (size_t(D) + 2) * sizeof(float) + 256;
}

// Dense split-KV pass over k,v [B,Hk,S,D] (bf16/fp8) writing `nsplit_here` splits at
// offset `split_offset` of `part`. Returns the number of splits it will use via
// dense_split_count (call it first to size the buffer).
int dense_split_count(int64_t B, int64_t Hq, int64_t Hk, int64_t S, int64_t D, int target_ctas);
// pdl: launch as a programmatic dependent of the previous kernel in the stream (which
// must not write what this pass reads); the pass waits for that kernel before it exits.
int launch_dense_partials(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, float scaling,
                          const Partials& part, int split_offset, int nsplit_here, cudaStream_t st,
                          bool pdl = false);
// One dense split per (b, KV head, head chunk) over k,v, launched as a programmatic
// dependent of the pass that fills slots [0, split_offset) of `part`: each CTA waits for
// that pass, then merges those slots with its own result and writes `out` (no combine
// kernel). Needs D % 4 == 0.
int launch_dense_merge(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, float scaling,
                       const Partials& part, int split_offset, const bd_tensor* out, cudaStream_t st);

// Final merge of all splits in `part` into out [B,Hq,D] (bf16/f16/f32). pdl: launch as a
// programmatic dependent; the kernel waits for its predecessor before reading partials.
// Merge of the split partials exported as one (m, l, o) per row: m,l [B*Hq] (m in natural-log
// units of scaling*q.k), o [B*Hq,D] un-normalised — the shard partial of a split-KV exchange.
int launch_combine_export(const Partials& part, int B, int Hq, int D, float* em, float* el, float* eo,
                          cudaStream_t st, bool pdl);
int launch_combine(const Partials& part, int B, int Hq, int D, const bd_tensor* out, cudaStream_t st,
                   bool pdl = false);

// Launch `kern` with the programmatic stream serialization attribute, any parameter list.
// The kernel may then start while the previous kernel in the stream is finishing, so it
// must call griddep_wait() before it reads or writes global memory.
template <typename... Params, typename... Args>
int launch_pdl(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, const char* what,
               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_check(cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...), what);
}

// Launch `kern` with the programmatic stream serialization attribute.
template <typename Params>
int launch_programmatic(void (*kern)(Params), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                        const Params& prm, const char* what) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_check(cudaLaunchKernelEx(&cfg, kern, prm), what);
}

}  // namespace bd
