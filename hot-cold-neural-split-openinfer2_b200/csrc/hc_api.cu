// Library identity and small device queries of the C ABI.
#include <cstring>

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

// ---------------------------------------------------------------------------
// Exchange buffers of the tensor-parallel stack: one cudaMalloc'd block per
// GPU (so its IPC handle maps the block itself), shared with the other ranks
// through CUDA IPC handles.
// ---------------------------------------------------------------------------
extern "C" int hc_tp_alloc(int64_t bytes, void** ptr) {
  if (bytes <= 0 || !ptr) return HC_ERR_ARG;
  *ptr = nullptr;
  if (cudaMalloc(ptr, (size_t)bytes) != cudaSuccess) return HC_ERR_CUDA;
  if (cudaMemset(*ptr, 0, (size_t)bytes) != cudaSuccess) return HC_ERR_CUDA;
  return HC_OK;
}

extern "C" int hc_tp_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? HC_OK : HC_ERR_CUDA; }

extern "C" int hc_ipc_get_handle(void* ptr, uint8_t* handle) {
  if (!ptr || !handle) return HC_ERR_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return HC_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  return HC_OK;
}

extern "C" int hc_ipc_open(const uint8_t* handle, void** ptr) {
  if (!handle || !ptr) return HC_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

extern "C" int hc_ipc_close(void* ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? HC_OK : HC_ERR_CUDA; }
