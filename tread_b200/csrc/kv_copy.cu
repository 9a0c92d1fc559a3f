// Block-store tier transfers: pinned host <-> HBM copies on a caller-chosen (side) stream.
//
// Replaces the synchronous `.to("cpu").pin_memory()` spill (tread/store.py:111, a pageable
// copy then a second pinned copy, both on the current stream) and the `.to(device,
// non_blocking=True)` fetch (tread/store.py:75-76) with one DMA-engine copy each, issued on a
// stream the store dedicates to transfers so that they overlap kernels on the compute
// stream. The row-strided variants move one block's slice of an assembled
// [L, Hkv, T, D] cache (L*Hkv rows of n*D elements at a pitch of T*D).
#include "common.cuh"

namespace tread {
namespace {

enum Side { kHost, kDevice };

int check_ptr(const void* p, Side want, const char* what) {
  cudaPointerAttributes a;
  cudaError_t e = cudaPointerGetAttributes(&a, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("%s: cudaPointerGetAttributes: %s", what, cudaGetErrorString(e));
    return TREAD_ERR_CUDA;
  }
  if (want == kHost && a.type != cudaMemoryTypeHost) {
    set_error("%s: host buffer is not page-locked (pinned) memory", what);
    return TREAD_ERR_INVALID;
  }
  if (want == kDevice && a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged) {
    set_error("%s: device buffer is not device memory", what);
    return TREAD_ERR_INVALID;
  }
  return TREAD_OK;
}

}  // namespace
}  // namespace tread

extern "C" int tread_kv_fetch(void* dst_device, const void* src_host, size_t bytes, tread_stream_t stream) {
  using namespace tread;
  if (bytes == 0) return TREAD_OK;
  TREAD_CHECK_ARG(dst_device && src_host, "kv_fetch: null pointer");
  int rc = check_ptr(src_host, kHost, "kv_fetch src");
  if (rc) return rc;
  rc = check_ptr(dst_device, kDevice, "kv_fetch dst");
  if (rc) return rc;
  TREAD_CHECK_CUDA(cudaMemcpyAsync(dst_device, src_host, bytes, cudaMemcpyHostToDevice,
                                   reinterpret_cast<cudaStream_t>(stream)));
  return TREAD_OK;
}

extern "C" int tread_kv_spill(void* dst_host, const void* src_device, size_t bytes, tread_stream_t stream) {
  using namespace tread;
  if (bytes == 0) return TREAD_OK;
  TREAD_CHECK_ARG(dst_host && src_device, "kv_spill: null pointer");
  int rc = check_ptr(dst_host, kHost, "kv_spill dst");
  if (rc) return rc;
  rc = check_ptr(src_device, kDevice, "kv_spill src");
  if (rc) return rc;
  TREAD_CHECK_CUDA(cudaMemcpyAsync(dst_host, src_device, bytes, cudaMemcpyDeviceToHost,
                                   reinterpret_cast<cudaStream_t>(stream)));
  return TREAD_OK;
}

extern "C" int tread_kv_fetch_rows(void* dst_device, size_t dst_pitch, const void* src_host, size_t src_pitch,
                                   size_t row_bytes, size_t nrows, tread_stream_t stream) {
  using namespace tread;
  if (row_bytes == 0 || nrows == 0) return TREAD_OK;
  TREAD_CHECK_ARG(dst_device && src_host, "kv_fetch_rows: null pointer");
  TREAD_CHECK_ARG(row_bytes <= dst_pitch && row_bytes <= src_pitch, "kv_fetch_rows: row_bytes exceeds a pitch");
  int rc = check_ptr(src_host, kHost, "kv_fetch_rows src");
  if (rc) return rc;
  rc = check_ptr(dst_device, kDevice, "kv_fetch_rows dst");
  if (rc) return rc;
  TREAD_CHECK_CUDA(cudaMemcpy2DAsync(dst_device, dst_pitch, src_host, src_pitch, row_bytes, nrows,
                                     cudaMemcpyHostToDevice, reinterpret_cast<cudaStream_t>(stream)));
  return TREAD_OK;
}

extern "C" int tread_kv_spill_rows(void* dst_host, size_t dst_pitch, const void* src_device, size_t src_pitch,
                                   size_t row_bytes, size_t nrows, tread_stream_t stream) {
  using namespace tread;
  if (row_bytes == 0 || nrows == 0) return TREAD_OK;
  TREAD_CHECK_ARG(dst_host && src_device, "kv_spill_rows: null pointer");
  TREAD_CHECK_ARG(row_bytes <= dst_pitch && row_bytes <= src_pitch, "kv_spill_rows: row_bytes exceeds a pitch");
  int rc = check_ptr(dst_host, kHost, "kv_spill_rows dst");
  if (rc) return rc;
  rc = check_ptr(src_device, kDevice, "kv_spill_rows src");
  if (rc) return rc;
  TREAD_CHECK_CUDA(cudaMemcpy2DAsync(dst_host, dst_pitch, src_device, src_pitch, row_bytes, nrows,
                                     cudaMemcpyDeviceToHost, reinterpret_cast<cudaStream_t>(stream)));
  return TREAD_OK;
}
