// Library identity and small device queries of the C ABI.
#include "hc_common.cuh"

extern "C" int hc_version(void) { return HC_ABI_VERSION; }

extern "C" const char* hc_status_string(int status) {
  if (status == HC_OK) return "ok";
  if (status & HC_ERR_ARG) return "invalid argument";
  if (status & HC_ERR_CUDA) return "CUDA runtime error";
  if (status & HC_ERR_RANGE) return "index out of range";
  if (status & HC_ERR_TIMEOUT) return "bounded wait expired";
  if (status & HC_ERR_UNSUPPORTED) return "unsupported shape or mode";
  return "unknown status";
}

extern "C" int hc_device_sm_count(void) {
  int n = 0, dev = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) return -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  return sms;
}
