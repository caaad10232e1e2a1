// Library state of libhsd: the thread-local last error, the ABI version and the
// device status words of every translation unit.
#include <cstdarg>
#include <cstdio>

#include "hsd_common.cuh"

namespace hsd {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

}  // namespace hsd

// status readers defined by HSD_DEFINE_STATUS in the kernel translation units
int hsd_read_status_decode(int* out, cudaStream_t st);
int hsd_read_status_prefill(int* out, cudaStream_t st);
int hsd_read_status_gemm(int* out, cudaStream_t st);
int hsd_read_status_up(int* out, cudaStream_t st);
int hsd_read_status_mamba(int* out, cudaStream_t st);
int hsd_read_status_norm(int* out, cudaStream_t st);
int hsd_read_status_attn(int* out, cudaStream_t st);
int hsd_read_status_qmma(int* out, cudaStream_t st);
int hsd_read_status_ep(int* out, cudaStream_t st);

extern "C" const char* hsd_last_error_string(void) { return hsd::g_last_error; }

extern "C" int hsd_abi_version(void) { return 1; }

extern "C" int hsd_device_status(int* status_out, void* stream) {
  if (!status_out) return hsd::set_error(HSD_ERR_ARG, "hsd_device_status: null output");
  cudaStream_t st = hsd::as_stream(stream);
  int first = HSD_OK;
  int (*readers[])(int*, cudaStream_t) = {hsd_read_status_decode, hsd_read_status_prefill,
                                                hsd_read_status_gemm, hsd_read_status_up,
                                                hsd_read_status_mamba, hsd_read_status_norm,
                                                hsd_read_status_attn, hsd_read_status_qmma,
                                                hsd_read_status_ep};
  for (auto rd : readers) {
    int v = HSD_OK;
    int rc = rd(&v, st);
    if (rc != HSD_OK) return rc;
    if (first == HSD_OK) first = v;
  }
  *status_out = first;
  return HSD_OK;
}
