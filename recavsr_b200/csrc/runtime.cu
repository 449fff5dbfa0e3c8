// Library-wide host support: last-error text, launch checks, TMA descriptor
// encoding and the device error word readout.
#include <cudaTypedefs.h>
#include <mutex>
#include <string>

#include "common.cuh"

namespace {
thread_local std::string g_last_error;
PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
std::once_flag g_encode_once;
}  // namespace

namespace rc {

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(RC_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return RC_OK;
}

int check_launch(cudaError_t launched, const char* what) {
  if (launched != cudaSuccess) {
    cudaGetLastError();   // clear the sticky-free launch error
    return set_error(RC_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(launched));
  }
  return check_launch(what);
}

int ensure_smem_attr(SmemAttrFlags& flags, const void* func, int bytes, const char* what) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(RC_ERR_CUDA, "%s: no usable current device", what);
  if (flags.set[dev]) return RC_OK;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) {
    cudaGetLastError();
    return set_error(RC_ERR_CUDA, "%s: cannot reserve %d bytes of shared memory on device %d", what, bytes, dev);
  }
  __sync_synchronize();
  flags.set[dev] = 1;
  return RC_OK;
}

int sm_count() {
  static int cache[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle, const char* what) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode_tiled) return set_error(RC_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable", what);
  if (reinterpret_cast<uintptr_t>(base) % 16)
    return set_error(RC_ERR_ARG, "%s: base address must be 16-byte aligned", what);
  for (int i = 0; i + 1 < rank; ++i)
    if (strides_bytes[i] % 16)
      return set_error(RC_ERR_ARG, "%s: stride %d (%llu bytes) is not a multiple of 16", what,
                       i + 1, (unsigned long long)strides_bytes[i]);
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode_tiled(map, dtype, (cuuint32_t)rank, base, (const cuuint64_t*)dims,
                              (const cuuint64_t*)strides_bytes, (const cuuint32_t*)box,
                              elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(RC_ERR_ARG, "%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
  return RC_OK;
}

}  // namespace rc

// Per-unit device error readers (defined in each kernel unit).
unsigned int rc_take_device_error_quant();
unsigned int rc_take_device_error_glue();
unsigned int rc_take_device_error_gemm_nvf4();
unsigned int rc_take_device_error_gemm_fp8();
unsigned int rc_take_device_error_attention();
unsigned int rc_take_device_error_decoder_attention();

extern "C" {

int rc_get_last_error(char* buf, size_t size) {
  if (!buf || !size) return (int)g_last_error.size();
  snprintf(buf, size, "%s", g_last_error.c_str());
  return (int)g_last_error.size();
}

int rc_read_device_error(unsigned int* word) {
  if (!word) return rc::set_error(RC_ERR_ARG, "rc_read_device_error: null output");
  unsigned int all[] = {rc_take_device_error_quant(), rc_take_device_error_glue(),
                        rc_take_device_error_gemm_nvf4(), rc_take_device_error_gemm_fp8(),
                        rc_take_device_error_attention(), rc_take_device_error_decoder_attention()};
  *word = 0;
  for (unsigned int v : all)
    if (v && !*word) *word = v;
  return RC_OK;
}

int rc_abi_version(void) { return 1; }

}  // extern "C"
