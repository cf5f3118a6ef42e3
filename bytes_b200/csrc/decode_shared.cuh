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

inline Partials carve_partials(void* ws, size_t rows, int nsplit, int D) {
  float* base = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
  Partials p;
  p.m = base;
  p.l = base + rows * nsplit;
  p.o = base + 2 * rows * nsplit;
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
int launch_dense_partials(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, float scaling,
                          const Partials& part, int split_offset, int nsplit_here, cudaStream_t st);

// Final merge of all splits in `part` into out [B,Hq,D] (bf16/f16/f32).
int launch_combine(const Partials& part, int B, int Hq, int D, const bd_tensor* out, cudaStream_t st);

}  // namespace bd
