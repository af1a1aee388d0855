// ff_lib.cu — the single translation unit of libfirefly_b200.so.
//
// One TU keeps the device status word (ff::g_status) a plain __device__
// variable of this module without relocatable device code.
#include "ff_common.cuh"
#include "ff_adamw8_dense.cuh"
#include "ff_dqt_adamw8.cuh"
#include "ff_gelu.cuh"
#include "ff_quant.cuh"
#include "ff_norm.cuh"
#include "ff_gemm_i8.cuh"

#ifndef FF_VERSION_STRING
#define FF_VERSION_STRING "firefly_b200 0.1.0 sm_100a"
#endif

extern "C" const char* ff_version(void) { return FF_VERSION_STRING; }

extern "C" const char* ff_last_error(void) { return ff::last_error_storage().c_str(); }

extern "C" int ff_num_sms(int* out) {
  FF_REQUIRE(out, FF_ERR_INVALID_ARG, "ff_num_sms: null pointer");
  int dev = 0;
  FF_CUDA_TRY(cudaGetDevice(&dev), "ff_num_sms");
  FF_CUDA_TRY(cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev), "ff_num_sms");
  return FF_OK;
}

extern "C" int ff_device_status(uint32_t* out, int clear) {
  FF_REQUIRE(out, FF_ERR_INVALID_ARG, "ff_device_status: null pointer");
  FF_CUDA_TRY(cudaDeviceSynchronize(), "ff_device_status sync");
  FF_CUDA_TRY(cudaMemcpyFromSymbol(out, ff::g_status, sizeof(uint32_t)), "ff_device_status read");
  if (clear) {
    const uint32_t zero = 0;
    FF_CUDA_TRY(cudaMemcpyToSymbol(ff::g_status, &zero, sizeof(uint32_t)), "ff_device_status clear");
  }
  return FF_OK;
}

extern "C" int ff_set_wait_limit_ns(uint64_t ns) {
  const uint64_t v = ns ? ns : ff::kWaitLimitNs;
  FF_CUDA_TRY(cudaMemcpyToSymbol(ff::g_wait_limit_ns, &v, sizeof(v)), "ff_set_wait_limit_ns");
  return FF_OK;
}

// ---------------------------------------------------------------------------
// ff_quant_dual_i8_noalloc: ff_quant_dual_i8 with its absmax workspace in a
// static device array of this library instead of caller-provided memory.
//
// The array (FF_NOALLOC_DUAL_MAX_ELEMS floats, 1 MiB) exists on every GPU that
// loads the library, for the life of the process.  Host code cannot use the
// symbol itself as a device address, so every call asks the runtime for the
// array's device address on the current device (cudaGetSymbolAddress: a query,
// no allocation).  Asking each time keeps the address right after a context
// reset, which reloads the module and can move the array.  Every call shares the
// array: ff_quant_dual_i8 clears the part it uses (the absmax accumulators must
// start at zero) with cudaMemsetAsync on the call's stream, so calls that overlap
// on the GPU would race on it.
// ---------------------------------------------------------------------------
static __device__ __align__(256) float g_noalloc_absmax[FF_NOALLOC_DUAL_MAX_ELEMS];

extern "C" int ff_quant_dual_i8_noalloc(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ldx,
                                        const float* row_colmul, float eps, int8_t* q_rows, int64_t ldq,
                                        float* s_rows, int8_t* q_cols_t, int64_t ldqt, float* s_cols,
                                        void* stream) {
  FF_REQUIRE(rows >= 0 && cols >= 0, FF_ERR_INVALID_ARG, "ff_quant_dual_i8_noalloc: rows=%lld cols=%lld",
             (long long)rows, (long long)cols);
  constexpr int64_t kMax = FF_NOALLOC_DUAL_MAX_ELEMS;
  FF_REQUIRE(rows <= kMax && cols <= kMax - rows, FF_ERR_UNSUPPORTED,
             "ff_quant_dual_i8_noalloc: rows=%lld + cols=%lld exceeds the built-in scratch of %lld elements; "
             "use ff_quant_dual_i8 with a workspace",
             (long long)rows, (long long)cols, (long long)kMax);
  void* addr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_absmax);
  if (e != cudaSuccess || addr == nullptr)
    return ff::set_error(FF_ERR_CUDA, "ff_quant_dual_i8_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
  return ff_quant_dual_i8(x, dtype, rows, cols, ldx, row_colmul, eps, q_rows, ldq, s_rows, q_cols_t, ldqt,
                          s_cols, static_cast<float*>(addr), stream);
}

// ---------------------------------------------------------------------------
// Device memory shared between the processes of one node (CUDA IPC): the data-parallel
// optimizer's weight and gradient arenas, which every rank's update kernel reads and writes
// over NVLink.  ff_ipc_alloc returns a whole cudaMalloc allocation (IPC handles name
// allocations); the handle (FF_IPC_HANDLE_BYTES bytes) is opened in another process with
// ff_ipc_open, which maps the allocation there and enables peer access.
// ---------------------------------------------------------------------------
static_assert(sizeof(cudaIpcMemHandle_t) == FF_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int ff_ipc_alloc(int64_t bytes, void** ptr) {
  FF_REQUIRE(ptr && bytes > 0, FF_ERR_INVALID_ARG, "ff_ipc_alloc: bytes=%lld", (long long)bytes);
  *ptr = nullptr;
  FF_CUDA_TRY(cudaMalloc(ptr, (size_t)bytes), "ff_ipc_alloc");
  return FF_OK;
}

extern "C" int ff_ipc_free(void* ptr) {
  if (ptr) FF_CUDA_TRY(cudaFree(ptr), "ff_ipc_free");
  return FF_OK;
}

extern "C" int ff_ipc_get_handle(void* ptr, uint8_t* handle) {
  FF_REQUIRE(ptr && handle, FF_ERR_INVALID_ARG, "ff_ipc_get_handle: null pointer");
  cudaIpcMemHandle_t h;
  FF_CUDA_TRY(cudaIpcGetMemHandle(&h, ptr), "ff_ipc_get_handle");
  memcpy(handle, &h, sizeof(h));
  return FF_OK;
}

extern "C" int ff_ipc_open(const uint8_t* handle, void** ptr) {
  FF_REQUIRE(handle && ptr, FF_ERR_INVALID_ARG, "ff_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  FF_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "ff_ipc_open");
  return FF_OK;
}

extern "C" int ff_ipc_close(void* ptr) {
  if (ptr) FF_CUDA_TRY(cudaIpcCloseMemHandle(ptr), "ff_ipc_close");
  return FF_OK;
}
