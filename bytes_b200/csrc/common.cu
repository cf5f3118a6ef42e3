// Host-side helpers shared by every entry point: error reporting and descriptor checks.
#include "common.cuh"

#include <cudaTypedefs.h>

#include <mutex>

namespace bd {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
  g_last_error = std::string(bd_status_name(status)) + ": " + msg;
  return status;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return BD_OK;
  // a launch that the runtime refused also left its code as the thread's last error; clear
  // it so the next call's launch check does not report this one's failure again
  (void)cudaGetLastError();
  return fail(BD_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

namespace {
using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda)
EncodeFn tensor_map_encoder() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(f);
  });
  return fn;
}
}  // namespace

bool encode_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* ptr, const cuuint64_t* dims,
                const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw) {
  const EncodeFn enc = tensor_map_encoder();
  if (!enc || rank < 1 || rank > 5) return false;
  const cuuint32_t es[5] = {1, 1, 1, 1, 1};
  return enc(m, dt, cuuint32_t(rank), const_cast<void*>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (sms[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    sms[dev] = v > 0 ? v : 148;
  }
  return sms[dev];
}

const char* dtype_name(int dt) {
  switch (dt) {
    case BD_F32: return "f32";
    case BD_F16: return "f16";
    case BD_BF16: return "bf16";
    case BD_F8E4M3: return "f8e4m3";
    case BD_U8: return "u8";
    case BD_I8: return "i8";
    case BD_I32: return "i32";
    case BD_I64: return "i64";
  }
  return "?";
}

std::string shape_str(const bd_tensor* t) {
  std::string s = "[";
  for (int i = 0; i < t->ndim; ++i) {
    s += std::to_string(t->shape[i]);
    if (i + 1 < t->ndim) s += ",";
  }
  return s + "]";
}

int check_tensor(const bd_tensor* t, const char* name, int ndim, int dtype) {
  if (!t) return fail(BD_ERR_NULL, std::string(name) + " descriptor is NULL");
  if (t->ndim != ndim)
    return fail(BD_ERR_SHAPE, std::string(name) + " must have " + std::to_string(ndim) +
                                  " dims, got " + std::to_string(t->ndim));
  if (dtype >= 0 && t->dtype != dtype)
    return fail(BD_ERR_DTYPE, std::string(name) + " must be " + dtype_name(dtype) + ", got " +
                                  dtype_name(t->dtype));
  int64_t numel = 1;
  for (int i = 0; i < ndim; ++i) {
    if (t->shape[i] < 0) return fail(BD_ERR_SHAPE, std::string(name) + " has a negative dim");
    numel *= t->shape[i];
  }
  if (numel > 0 && !t->data) return fail(BD_ERR_NULL, std::string(name) + " data pointer is NULL");
  return BD_OK;
}

int check_rows_aligned(const bd_tensor* t, const char* name, size_t align) {
  const size_t es = dtype_size(t->dtype);
  if (t->ndim > 0 && t->shape[t->ndim - 1] > 1 && t->stride[t->ndim - 1] != 1)
    return fail(BD_ERR_STRIDE, std::string(name) + " innermost dim must be contiguous");
  if (reinterpret_cast<uintptr_t>(t->data) % align)
    return fail(BD_ERR_ALIGN, std::string(name) + " base pointer not " + std::to_string(align) + "-byte aligned");
  for (int i = 0; i + 1 < t->ndim; ++i)
    if (t->shape[i] > 1 && (size_t(t->stride[i]) * es) % align)
      return fail(BD_ERR_ALIGN, std::string(name) + " stride of dim " + std::to_string(i) +
                                    " is not a multiple of " + std::to_string(align) + " bytes");
  return BD_OK;
}

}  // namespace bd

extern "C" {

int bd_abi_version(void) { return 1; }

long long bd_wait_timeouts(void) {
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  const long long a = bd::kivi_wait_timeouts(), b = bd::pq_wait_timeouts(), c = bd::merge_wait_timeouts(),
                  d = bd::exchange_wait_timeouts();
  return (a < 0 || b < 0 || c < 0 || d < 0) ? -1 : a + b + c + d;
}

const char* bd_status_name(int s) {
  switch (s) {
    case BD_OK: return "BD_OK";
    case BD_ERR_NULL: return "BD_ERR_NULL";
    case BD_ERR_DTYPE: return "BD_ERR_DTYPE";
    case BD_ERR_SHAPE: return "BD_ERR_SHAPE";
    case BD_ERR_STRIDE: return "BD_ERR_STRIDE";
    case BD_ERR_ALIGN: return "BD_ERR_ALIGN";
    case BD_ERR_WORKSPACE: return "BD_ERR_WORKSPACE";
    case BD_ERR_UNSUPPORTED: return "BD_ERR_UNSUPPORTED";
    case BD_ERR_CUDA: return "BD_ERR_CUDA";
    case BD_ERR_VALUE: return "BD_ERR_VALUE";
  }
  return "BD_ERR_UNKNOWN";
}

const char* bd_last_error(void) { return bd::g_last_error.c_str(); }

}  // extern "C"
