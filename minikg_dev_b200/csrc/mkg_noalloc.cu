// ind2ptr for callers that cannot allocate device memory.
//
// Callers such as a plain C or FFI host that holds only the device pointers it was handed
// (no device allocator of its own), or code that must not trigger an allocation on its
// path, cannot provide the workspace that mkg_ind2ptr needs.  mkg_ind2ptr_noalloc takes
// the same inputs and output but keeps its scratch (the per-row counts and the scan's
// temporary storage) in one file-scope device array, g_noalloc_scratch, of fixed size.
// Every GPU that loads this library holds that array until the process exits.
//
// In host code the array's name is only a host-side stand-in, not a device address, so the
// address is looked up with cudaGetSymbolAddress while the call's device is current.  The
// lookup is repeated on every call made outside a stream capture (after a cudaDeviceReset the
// module is loaded again and the array can move); a call made while its stream is being
// captured reuses the address of the last call outside a capture on that device, so the
// first call on a device should come before any stream capture.  All calls share the array
// and it keeps the last call's contents: the counts are cleared on every call, and calls
// that overlap on the GPU (for instance on two streams at once) race on it.
#include <mutex>

#include <cub/cub.cuh>

#include "mkg_common.cuh"

#define MKG_API extern "C" __attribute__((visibility("default")))

namespace mkg {
namespace {

constexpr int64_t kNoAllocMaxRows = MKG_NOALLOC_MAX_ROWS;
constexpr size_t kCountBytes = ((8 * (size_t)(kNoAllocMaxRows + 1)) + 255) & ~size_t(255);
constexpr size_t kTempBytes = 256 * 1024;

__device__ __align__(256) unsigned char g_noalloc_scratch[kCountBytes + kTempBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch for the current device: looked up again on every call
// outside a stream capture, taken from the last such lookup while `st` is capturing.
int noalloc_scratch(cudaStream_t st, void** out) {
  int dev = 0;
  MKG_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("ind2ptr_noalloc: device ordinal %d out of range", dev);
    return MKG_ERR_ARG;
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  MKG_CUDA(cudaStreamIsCapturing(st, &cap));
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (cap == cudaStreamCaptureStatusNone || g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return MKG_OK;
}

__global__ void noalloc_count_kernel(const int64_t* __restrict__ index, int64_t n, int64_t size,
                                     int64_t* __restrict__ cnt, unsigned* err) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = index[i];
    if (r < 0 || r >= size) { raise_flag(err, MKG_DEV_BAD_ENTRY); continue; }
    atomicAdd(reinterpret_cast<unsigned long long*>(cnt + r + 1), 1ull);
  }
}

}  // namespace
}  // namespace mkg

MKG_API int mkg_ind2ptr_noalloc(const int64_t* index, int64_t n, int64_t size, int64_t* ptr, unsigned* dev_err,
                                mkg_stream stream) {
  using namespace mkg;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if ((!index && n > 0) || !ptr) { set_error("ind2ptr_noalloc: null argument"); return MKG_ERR_ARG; }
  if (n < 0 || size < 0) { set_error("ind2ptr_noalloc: negative size"); return MKG_ERR_ARG; }
  if (size > kNoAllocMaxRows) {
    set_error("ind2ptr_noalloc: size %lld exceeds the static scratch limit of %lld rows; use mkg_ind2ptr "
              "with a caller-provided workspace", (long long)size, (long long)kNoAllocMaxRows);
    return MKG_ERR_CAPACITY;
  }
  size_t temp_need = 0;
  MKG_CUDA(cub::DeviceScan::InclusiveSum(nullptr, temp_need, (int64_t*)nullptr, (int64_t*)nullptr, (int)size));
  if (temp_need > kTempBytes) {
    set_error("ind2ptr_noalloc: scan needs %zu bytes of temporary storage, the static scratch has %zu", temp_need,
              kTempBytes);
    return MKG_ERR_CAPACITY;
  }
  void* base = nullptr;
  int rc = noalloc_scratch(st, &base);
  if (rc) return rc;
  int64_t* cnt = static_cast<int64_t*>(base);
  void* temp = static_cast<char*>(base) + kCountBytes;
  // the scratch keeps the previous call's counts: clear the part this call uses
  MKG_CUDA(cudaMemsetAsync(cnt, 0, sizeof(int64_t) * (size + 1), st));
  MKG_CUDA(cudaMemsetAsync(ptr, 0, sizeof(int64_t), st));
  if (n > 0) {
    noalloc_count_kernel<<<grid_for(n, 256, persistent_blocks(4)), 256, 0, st>>>(index, n, size, cnt, dev_err);
    MKG_LAUNCHED("noalloc_count_kernel");
  }
  if (size > 0) {
    size_t tb = kTempBytes;
    MKG_CUDA(cub::DeviceScan::InclusiveSum(temp, tb, cnt + 1, ptr + 1, (int)size, st));
  }
  return MKG_OK;
}
