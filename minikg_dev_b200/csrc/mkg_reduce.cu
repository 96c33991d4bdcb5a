// Reduce-by-key of sparse COO states: the coalescing behind the bridge reducers
// (sum_sparse3d_concat / sum_sp_3d, fastlog_bridge.py:17-42; max_sp_3d / sparse3d_max,
// model_mmDRUM_kernel_sp.py:184-270) on the device.
//
// Entries (key, value) are sorted by key with a stable LSD radix sort over the key's
// significant bits (equal keys keep their input order), runs of equal keys become one output
// entry each, in ascending key order:
//  * sum: the run's values added in fp64 and rounded once;
//  * max: the largest value; among equal largest values the run's first entry (the earliest
//    in input order) wins, through one packed 64-bit atomicMax per entry of
//    (order-preserving value bits << 32 | ~position in the sorted run order).
// inverse[i] = output index of input entry i (the gradient of a sum gathers through it) and
// arg[u] = the input entry that won output u (the gradient of a max scatters through it).
#include <cub/cub.cuh>

#include "mkg_common.cuh"

#define MKG_API extern "C" __attribute__((visibility("default")))

namespace mkg {
namespace {

size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

struct ReduceLayout {
  size_t skeys, idx, sidx, flags, acc, temp, total;
  size_t temp_bytes;
};

ReduceLayout reduce_layout(int64_t n) {
  ReduceLayout L{};
  size_t sort_b = 0, scan_b = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, sort_b, (const unsigned long long*)nullptr, (unsigned long long*)nullptr,
                                  (const int32_t*)nullptr, (int32_t*)nullptr, (int)n);
  cub::DeviceScan::InclusiveSum(nullptr, scan_b, (int64_t*)nullptr, (int64_t*)nullptr, (int)n);
  L.temp_bytes = std::max(sort_b, scan_b);
  size_t o = 0;
  L.skeys = o; o += a256(8 * (size_t)n);
  L.idx = o; o += a256(4 * (size_t)n);
  L.sidx = o; o += a256(4 * (size_t)n);
  L.flags = o; o += a256(8 * (size_t)n);
  L.acc = o; o += a256(8 * (size_t)n);  // fp64 sums or packed maxima per run
  L.temp = o; o += a256(L.temp_bytes);
  L.total = o;
  return L;
}

__global__ void iota_check_kernel(const int64_t* __restrict__ keys, int64_t n, int32_t* __restrict__ idx,
                                  unsigned long long* __restrict__ acc, unsigned* err) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    idx[i] = static_cast<int32_t>(i);
    acc[i] = 0ull;
    if (keys[i] < 0) raise_flag(err, MKG_DEV_BAD_KEY);
  }
}

__global__ void run_heads_kernel(const unsigned long long* __restrict__ skeys, int64_t n, int64_t* __restrict__ flags) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    flags[i] = (i == 0 || skeys[i] != skeys[i - 1]) ? 1 : 0;
}

// flags now holds the inclusive run count: run of sorted entry i = flags[i] - 1
__global__ void run_reduce_kernel(const unsigned long long* __restrict__ skeys, const int32_t* __restrict__ sidx,
                                  const int64_t* __restrict__ runs, const float* __restrict__ vals, int64_t n, int mode,
                                  unsigned long long* __restrict__ acc, int64_t* __restrict__ out_keys,
                                  int64_t* __restrict__ inverse) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t u = runs[i] - 1;
    const int32_t src = sidx[i];
    if (i == 0 || runs[i - 1] != runs[i]) out_keys[u] = static_cast<int64_t>(skeys[i]);
    if (inverse) inverse[src] = u;
    const float v = vals[src];
    if (mode == 0) {
      atomicAdd(reinterpret_cast<double*>(acc) + u, static_cast<double>(v));
    } else {
      atomicMax(acc + u, pack_value_rank(v, static_cast<uint32_t>(i)));
    }
  }
}

__global__ void run_finish_kernel(const unsigned long long* __restrict__ acc, const int32_t* __restrict__ sidx,
                                  const int64_t* __restrict__ runs, const float* __restrict__ vals, int64_t n, int mode,
                                  float* __restrict__ out_vals, int64_t* __restrict__ arg) {
  const int64_t U = runs[n - 1];
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < U; u += (int64_t)gridDim.x * blockDim.x) {
    if (mode == 0) {
      out_vals[u] = static_cast<float>(reinterpret_cast<const double*>(acc)[u]);
    } else {
      const uint32_t pos = packed_rank(acc[u]);
      const int32_t src = sidx[pos];
      out_vals[u] = vals[src];
      if (arg) arg[u] = src;
    }
  }
}

}  // namespace
}  // namespace mkg

using namespace mkg;

MKG_API size_t mkg_reduce_by_key_workspace_bytes(int64_t n) {
  if (n <= 0) return 0;
  return reduce_layout(n).total;
}

MKG_API int mkg_reduce_by_key(const int64_t* keys, const float* vals, int64_t n, int32_t mode, int32_t key_bits,
                              int64_t* out_keys, float* out_vals, int64_t* count_out, int64_t* inverse, int64_t* arg,
                              void* workspace, size_t workspace_bytes, unsigned* dev_err, mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(mode == 0 || mode == 1, "reduce_by_key: mode must be 0 (sum) or 1 (max)");
  MKG_REQUIRE(n >= 0 && n < INT32_MAX, "reduce_by_key: %lld entries (at most 2^31 - 1)", (long long)n);
  MKG_REQUIRE(key_bits >= 1 && key_bits <= 63, "reduce_by_key: key_bits must lie in [1, 63]");
  MKG_REQUIRE(count_out, "reduce_by_key: null count");
  if (n == 0) {
    MKG_CUDA(cudaMemsetAsync(count_out, 0, sizeof(int64_t), st));
    return MKG_OK;
  }
  MKG_REQUIRE(keys && vals && out_keys && out_vals && workspace, "reduce_by_key: null argument");
  const ReduceLayout L = reduce_layout(n);
  MKG_REQUIRE(workspace_bytes >= L.total, "reduce_by_key: workspace too small");
  char* base = static_cast<char*>(workspace);
  auto* skeys = reinterpret_cast<unsigned long long*>(base + L.skeys);
  auto* idx = reinterpret_cast<int32_t*>(base + L.idx);
  auto* sidx = reinterpret_cast<int32_t*>(base + L.sidx);
  auto* flags = reinterpret_cast<int64_t*>(base + L.flags);
  auto* acc = reinterpret_cast<unsigned long long*>(base + L.acc);
  void* temp = base + L.temp;
  const int grid = grid_for(n, 256, persistent_blocks(8));
  iota_check_kernel<<<grid, 256, 0, st>>>(keys, n, idx, acc, dev_err);
  MKG_LAUNCHED("iota_check_kernel");
  size_t tb = L.temp_bytes;
  MKG_CUDA(cub::DeviceRadixSort::SortPairs(temp, tb, reinterpret_cast<const unsigned long long*>(keys), skeys, idx,
                                           sidx, (int)n, 0, key_bits, st));
  run_heads_kernel<<<grid, 256, 0, st>>>(skeys, n, flags);
  MKG_LAUNCHED("run_heads_kernel");
  tb = L.temp_bytes;
  MKG_CUDA(cub::DeviceScan::InclusiveSum(temp, tb, flags, flags, (int)n, st));
  run_reduce_kernel<<<grid, 256, 0, st>>>(skeys, sidx, flags, vals, n, mode, acc, out_keys, inverse);
  MKG_LAUNCHED("run_reduce_kernel");
  run_finish_kernel<<<grid, 256, 0, st>>>(acc, sidx, flags, vals, n, mode, out_vals, arg);
  MKG_LAUNCHED("run_finish_kernel");
  MKG_CUDA(cudaMemcpyAsync(count_out, flags + (n - 1), sizeof(int64_t), cudaMemcpyDeviceToDevice, st));
  return MKG_OK;
}
