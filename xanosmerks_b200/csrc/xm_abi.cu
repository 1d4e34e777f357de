// Host-side plumbing of the C ABI: error reporting and type geometry.
#include <cstdarg>
#include <cstdio>

#include "xm_qtypes.cuh"

namespace {
thread_local char g_last_error[512] = "";
}

// Device-side error word (per device): bounded waits that gave up set a bit.
__device__ int g_xm_device_error = 0;

int xm_set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int xm_check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return XM_OK;
}

bool host_qtype_geometry(int qtype, int* qk, int* rec) {
  int a = 0, b = 0;
  switch (qtype) {
    case T_F32: a = 1; b = 4; break;
    case T_F16: a = 1; b = 2; break;
    case T_BF16: a = 1; b = 2; break;
    case T_I8: a = 1; b = 1; break;
    case T_I16: a = 1; b = 2; break;
    case T_I32: a = 1; b = 4; break;
    case T_I64: a = 1; b = 8; break;
    case T_Q4_0: a = QT<T_Q4_0>::QK; b = QT<T_Q4_0>::REC; break;
    case T_Q4_1: a = QT<T_Q4_1>::QK; b = QT<T_Q4_1>::REC; break;
    case T_Q5_0: a = QT<T_Q5_0>::QK; b = QT<T_Q5_0>::REC; break;
    case T_Q5_1: a = QT<T_Q5_1>::QK; b = QT<T_Q5_1>::REC; break;
    case T_Q8_0: a = QT<T_Q8_0>::QK; b = QT<T_Q8_0>::REC; break;
    case T_Q8_1: a = QT<T_Q8_1>::QK; b = QT<T_Q8_1>::REC; break;
    case T_Q2_K: a = QT<T_Q2_K>::QK; b = QT<T_Q2_K>::REC; break;
    case T_Q3_K: a = QT<T_Q3_K>::QK; b = QT<T_Q3_K>::REC; break;
    case T_Q4_K: a = QT<T_Q4_K>::QK; b = QT<T_Q4_K>::REC; break;
    case T_Q5_K: a = QT<T_Q5_K>::QK; b = QT<T_Q5_K>::REC; break;
    case T_Q6_K: a = QT<T_Q6_K>::QK; b = QT<T_Q6_K>::REC; break;
    case T_Q8_K: a = QT<T_Q8_K>::QK; b = QT<T_Q8_K>::REC; break;
    default: return false;
  }
  if (qk) *qk = a;
  if (rec) *rec = b;
  return true;
}

extern "C" {

int xm_abi_version(void) { return 2; }

const char* xm_last_error(void) { return g_last_error; }

int xm_device_status(int clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_xm_device_error, sizeof(int));
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "device_status: %s", cudaGetErrorString(e));
  if (clear && v) {
    const int z = 0;
    e = cudaMemcpyToSymbol(g_xm_device_error, &z, sizeof(int));
    if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "device_status: %s", cudaGetErrorString(e));
  }
  return v;
}

int xm_device_status_async(int* h_word, void* stream) {
  if (!h_word) return xm_set_error(XM_ERR_INVALID, "device_status_async: null destination");
  cudaError_t e = cudaMemcpyFromSymbolAsync(h_word, g_xm_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost,
                                            (cudaStream_t)stream);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "device_status_async: %s", cudaGetErrorString(e));
  return XM_OK;
}

int xm_qtype_info(int qtype, int* qk, int* record_bytes) {
  if (!host_qtype_geometry(qtype, qk, record_bytes))
    return xm_set_error(XM_ERR_UNSUPPORTED, "type id %d is not supported", qtype);
  return XM_OK;
}

}  // extern "C"
