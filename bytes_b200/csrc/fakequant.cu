// Asymmetric uniform fake-quantisation (quantize then dequantize) over one axis.
//
// Follows _asym_uniform_fakequant (src/quantization.py:432-442 of saifmb0/bytes), the
// arithmetic of KIVIQuantizer.quantize_key / quantize_value (:468-501):
//   xmin, xmax over the group axis; scale = clamp(xmax - xmin, 1e-8) / (levels - 1)
//   q = clamp(round_half_even((x - xmin) / scale), 0, levels - 1); y = q * scale + xmin
// Every step rounds like the reference's tensor ops in the input dtype (fp32, or bf16 /
// f16 after each op), with no fused multiply-add, so outputs are bit-identical to the
// reference run on a CUDA device. There PyTorch divides a tensor by a Python number as a
// multiplication by the number's fp32 reciprocal (formed on the host; for bf16 / f16 the
// product is taken in fp32 and rounded), so the scale is range * fp32(1/(levels-1)); the
// CPU run of the same expression divides and differs in the last bit of some scales.
#include "common.cuh"

namespace bd {
namespace {

template <typename T>
__device__ __forceinline__ float rnd(float x) { return to_f32<T>(from_f32<T>(x)); }
template <>
__device__ __forceinline__ float rnd<float>(float x) { return x; }

struct FqParams {
  const void* x; int64_t s[5];   // strides of (o0, o1, o2, glen, inner)
  int64_t n[5];                  // sizes
  void* y;                       // contiguous output, same logical shape
  int levels;
  float rcp;                     // fp32 1/(levels-1), formed on the host
};

template <typename T>
__global__ void fakequant_kernel(const FqParams p) {
  const int64_t col = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;  // (o0,o1,o2,inner)
  const int64_t ncol = p.n[0] * p.n[1] * p.n[2] * p.n[4];
  if (col >= ncol) return;
  const int64_t in = col % p.n[4];
  int64_t r = col / p.n[4];
  const int64_t i2 = r % p.n[2]; r /= p.n[2];
  const int64_t i1 = r % p.n[1], i0 = r / p.n[1];
  const T* x = static_cast<const T*>(p.x) + i0 * p.s[0] + i1 * p.s[1] + i2 * p.s[2] + in * p.s[4];
  T* y = static_cast<T*>(p.y) + (((i0 * p.n[1] + i1) * p.n[2] + i2) * p.n[3]) * p.n[4] + in;
  const int64_t gl = p.n[3];
  float lo = INFINITY, hi = -INFINITY;
  for (int64_t e = 0; e < gl; ++e) {
    const float v = to_f32<T>(x[e * p.s[3]]);
    lo = fminf(lo, v);
    hi = fmaxf(hi, v);
  }
  const float L = float(p.levels - 1);
  const float sc = rnd<T>(__fmul_rn(rnd<T>(fmaxf(rnd<T>(__fsub_rn(hi, lo)), rnd<T>(1e-8f))), p.rcp));
  for (int64_t e = 0; e < gl; ++e) {
    const float v = to_f32<T>(x[e * p.s[3]]);
    float q = rintf(rnd<T>(__fdiv_rn(rnd<T>(__fsub_rn(v, lo)), sc)));
    q = fminf(fmaxf(q, 0.f), L);
    y[e * p.n[4]] = from_f32<T>(__fadd_rn(rnd<T>(__fmul_rn(q, sc)), lo));
  }
}

}  // namespace
}  // namespace bd

extern "C" {

int bd_asym_fakequant(const bd_tensor* x, int levels, const bd_tensor* y, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if (!x) return fail(BD_ERR_NULL, "x is NULL");
  if ((rc = check_tensor(x, "x", 5)) || (rc = check_tensor(y, "y", 5, x->dtype))) return rc;
  if (levels < 2) return fail(BD_ERR_VALUE, "levels must be >= 2");
  if (x->dtype != BD_F32 && x->dtype != BD_BF16 && x->dtype != BD_F16) return fail(BD_ERR_DTYPE, "x must be f32/bf16/f16");
  int64_t s = 1;
  for (int i = 4; i >= 0; --i) {
    if (y->shape[i] != x->shape[i]) return fail(BD_ERR_SHAPE, "y must have x's shape");
    if (y->shape[i] > 1 && y->stride[i] != s) return fail(BD_ERR_STRIDE, "y must be contiguous");
    s *= y->shape[i];
  }
  FqParams p{};
  p.x = x->data; p.y = y->data; p.levels = levels;
  p.rcp = 1.0f / float(levels - 1);
  for (int i = 0; i < 5; ++i) { p.s[i] = x->stride[i]; p.n[i] = x->shape[i]; }
  const int64_t ncol = p.n[0] * p.n[1] * p.n[2] * p.n[4];
  if (ncol == 0 || p.n[3] == 0) return BD_OK;
  const unsigned blocks = unsigned((ncol + 255) / 256);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (x->dtype == BD_F32) fakequant_kernel<float><<<blocks, 256, 0, st>>>(p);
  else if (x->dtype == BD_BF16) fakequant_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(p);
  else fakequant_kernel<__half><<<blocks, 256, 0, st>>>(p);
  return cuda_check(cudaGetLastError(), "fakequant_kernel launch");
}

}  // extern "C"
