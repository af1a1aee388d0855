// ff_lib.cu — the single translation unit of libfirefly_b200.so.
//
// One TU keeps the device status word (ff::g_status) a plain __device__
// variable of this module without relocatable device code.
#include "ff_common.cuh"
#include "ff_dqt_adamw8.cuh"
#include "ff_gemm_i8.cuh"
#include "ff_quant.cuh"

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
