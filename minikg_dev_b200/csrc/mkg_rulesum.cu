// Sum (or max) over rules of a hop loop's final state without a full sort: sum_sp_3d
// (fastlog_bridge.py:17-23) and max_sp_3d (model_mmDRUM_kernel_sp.py:184-236) on a state in
// entity-major order (ascending entity, then row b * L + l), the order the key-slab engine
// emits.  There the L rules of one (entity, query) pair are adjacent, so:
//  1. run heads: entry i starts a run when its (e, b) differs from entry i - 1's; an inclusive
//     scan numbers the runs (their (e, b) ascend entity-major);
//  2. each run head folds its run in rule order (fp32 sum, l ascending, as a sequential CPU
//     coalesce adds them; or the maximum) into run r = its number;
//  3. one stable radix pass over the runs' query b (the bits of B) puts them in (b, e) order;
//  4. the result keys b * E + e and values come out in that order, and every entry learns its
//     output position (the backward gathers the result's gradient through it).
// No host synchronisation: the run count stays on the device; the sort runs over all n slots,
// runs past the count carrying the sentinel query B (sorted last).
#include <cub/cub.cuh>

#include "mkg_common.cuh"

#define MKG_API extern "C" __attribute__((visibility("default")))

namespace mkg {
namespace {

size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

struct RuleSumLayout {
  size_t scan, run_b, run_e, run_v, sorted_b, iota, perm, pos, count, temp, total;
  size_t temp_bytes;
};

RuleSumLayout rule_sum_layout(int64_t n) {
  RuleSumLayout L{};
  size_t sort_b = 0, scan_b = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, sort_b, (const int32_t*)nullptr, (int32_t*)nullptr,
                                  (const int32_t*)nullptr, (int32_t*)nullptr, (int)n);
  cub::DeviceScan::InclusiveSum(nullptr, scan_b, (int32_t*)nullptr, (int32_t*)nullptr, (int)n);
  L.temp_bytes = sort_b > scan_b ? sort_b : scan_b;
  size_t o = 0;
  L.scan = o; o += a256(4 * (size_t)n);      // run heads, then run numbers + 1
  L.run_b = o; o += a256(4 * (size_t)n);     // query of each run (B past the count)
  L.run_e = o; o += a256(8 * (size_t)n);     // entity of each run
  L.run_v = o; o += a256(4 * (size_t)n);     // value of each run
  L.sorted_b = o; o += a256(4 * (size_t)n);
  L.iota = o; o += a256(4 * (size_t)n);
  L.perm = o; o += a256(4 * (size_t)n);      // sorted position -> run
  L.pos = o; o += a256(4 * (size_t)n);       // run -> sorted position
  L.count = o; o += a256(8);
  L.temp = o; o += a256(L.temp_bytes);
  L.total = o;
  return L;
}

// entity e and query b of a key (b * L + l) * E + e: one 64-bit division, the row's division
// by L in 32 bits when the row fits
__device__ __forceinline__ void split_key(int64_t key, const FastDiv& E, int64_t L, int64_t& e, int64_t& b) {
  const int64_t q = E.div(key);
  e = key - q * E.d;
  b = (q <= 0x7fffffff && L <= 0x7fffffff) ? (int64_t)((uint32_t)q / (uint32_t)L) : q / L;
}

// (e, b) of an entry as one ascending composite (entity-major order of runs)
__device__ __forceinline__ int64_t run_code(int64_t key, const FastDiv& E, int64_t L, int64_t B) {
  int64_t e, b;
  split_key(key, E, L, e, b);
  return e * B + b;
}

__global__ void rule_heads_kernel(const int64_t* __restrict__ keys, int64_t n, FastDiv E, int64_t L, int64_t B,
                                  int32_t* __restrict__ head, int32_t* __restrict__ run_b, int32_t* __restrict__ iota,
                                  unsigned* err) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = keys[i];
    run_b[i] = static_cast<int32_t>(B);  // sentinel: overwritten for the runs that exist
    iota[i] = static_cast<int32_t>(i);
    int64_t e = 0, b = 0;
    if (k >= 0) split_key(k, E, L, e, b);
    if (k < 0 || b >= B) {
      raise_flag(err, MKG_DEV_BAD_KEY);
      head[i] = 0;
      continue;
    }
    int32_t h = 1;
    if (i > 0) {
      const int64_t kp = keys[i - 1];
      const int64_t c = e * B + b, cp = kp >= 0 ? run_code(kp, E, L, B) : -1;
      if (c == cp) h = 0;
      else if (c < cp) raise_flag(err, MKG_DEV_BAD_KEY);  // not entity-major: runs would split
    }
    head[i] = h;
  }
}

// scan[i] = number of runs up to and including entry i; a head folds its run
template <bool MAX>
__global__ void rule_runs_kernel(const int64_t* __restrict__ keys, const float* __restrict__ vals, int64_t n,
                                 FastDiv E, int64_t L, int64_t B, const int32_t* __restrict__ scan,
                                 int32_t* __restrict__ run_b, int64_t* __restrict__ run_e,
                                 float* __restrict__ run_v, int64_t* __restrict__ count) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    if (i == n - 1) *count = scan[i];
    const int32_t r = scan[i] - 1;
    if (r < 0 || (i > 0 && scan[i - 1] == scan[i])) continue;  // not a run head
    // the run is every following entry with the same run number (a bad key, flagged by the
    // heads pass, would fold into the run before it)
    float acc = vals[i];
    for (int64_t j = i + 1; j < n && scan[j] == scan[i]; ++j) acc = MAX ? fmaxf(acc, vals[j]) : __fadd_rn(acc, vals[j]);
    int64_t e, b;
    split_key(keys[i], E, L, e, b);
    run_b[r] = static_cast<int32_t>(b);
    run_e[r] = e;
    run_v[r] = acc;
  }
}

__global__ void rule_out_kernel(const int32_t* __restrict__ perm, const int32_t* __restrict__ run_b,
                                const int64_t* __restrict__ run_e, const float* __restrict__ run_v,
                                const int64_t* __restrict__ count, int64_t n, int64_t E,
                                int64_t* __restrict__ out_keys, float* __restrict__ out_vals,
                                int32_t* __restrict__ pos) {
  const int64_t c = *count;
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < c && j < n;
       j += (int64_t)gridDim.x * blockDim.x) {
    const int32_t r = perm[j];
    out_keys[j] = (int64_t)run_b[r] * E + run_e[r];
    out_vals[j] = run_v[r];
    pos[r] = static_cast<int32_t>(j);
  }
}

__global__ void rule_entry_pos_kernel(const int32_t* __restrict__ scan, const int32_t* __restrict__ pos, int64_t n,
                                      int64_t* __restrict__ out_pos) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int32_t r = scan[i] - 1;
    out_pos[i] = r >= 0 ? pos[r] : -1;
  }
}

int bits_for(int64_t v) {
  int b = 1;
  while (b < 31 && (int64_t(1) << b) <= v) ++b;
  return b;
}

}  // namespace
}  // namespace mkg

using namespace mkg;

MKG_API size_t mkg_rule_sum_workspace_bytes(int64_t n) { return n > 0 ? rule_sum_layout(n).total : 0; }

MKG_API int mkg_rule_sum(const int64_t* keys, const float* vals, int64_t n, int64_t E, int64_t L, int64_t B,
                         int32_t mode, int64_t* out_keys, float* out_vals, int64_t* out_pos, int64_t* count_out,
                         void* workspace, size_t workspace_bytes, unsigned* dev_err, mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(n >= 0 && E >= 1 && L >= 1 && B >= 1 && B < (int64_t(1) << 30) && (mode == 0 || mode == 1),
              "rule_sum: bad arguments");
  MKG_REQUIRE(n < INT32_MAX, "rule_sum: %lld entries exceed the scan limit", (long long)n);
  MKG_REQUIRE(count_out, "rule_sum: null count");
  if (n == 0) {
    MKG_CUDA(cudaMemsetAsync(count_out, 0, sizeof(int64_t), st));
    return MKG_OK;
  }
  MKG_REQUIRE(keys && vals && out_keys && out_vals && workspace, "rule_sum: null argument");
  const RuleSumLayout Ly = rule_sum_layout(n);
  MKG_REQUIRE(workspace_bytes >= Ly.total, "rule_sum: workspace too small");
  char* w = static_cast<char*>(workspace);
  auto* scan = reinterpret_cast<int32_t*>(w + Ly.scan);
  auto* run_b = reinterpret_cast<int32_t*>(w + Ly.run_b);
  auto* run_e = reinterpret_cast<int64_t*>(w + Ly.run_e);
  auto* run_v = reinterpret_cast<float*>(w + Ly.run_v);
  auto* sorted_b = reinterpret_cast<int32_t*>(w + Ly.sorted_b);
  auto* iota = reinterpret_cast<int32_t*>(w + Ly.iota);
  auto* perm = reinterpret_cast<int32_t*>(w + Ly.perm);
  auto* pos = reinterpret_cast<int32_t*>(w + Ly.pos);
  auto* count = reinterpret_cast<int64_t*>(w + Ly.count);
  void* temp = w + Ly.temp;
  size_t tb = Ly.temp_bytes;
  const int grid = grid_for(n, 256, persistent_blocks(8));
  const FastDiv fe = FastDiv::of(E);
  rule_heads_kernel<<<grid, 256, 0, st>>>(keys, n, fe, L, B, scan, run_b, iota, dev_err);
  MKG_LAUNCHED("rule_heads_kernel");
  MKG_CUDA(cub::DeviceScan::InclusiveSum(temp, tb, scan, scan, (int)n, st));
  if (mode == 1)
    rule_runs_kernel<true><<<grid, 256, 0, st>>>(keys, vals, n, fe, L, B, scan, run_b, run_e, run_v, count);
  else
    rule_runs_kernel<false><<<grid, 256, 0, st>>>(keys, vals, n, fe, L, B, scan, run_b, run_e, run_v, count);
  MKG_LAUNCHED("rule_runs_kernel");
  // stable: runs of one query keep their ascending-entity order
  MKG_CUDA(cub::DeviceRadixSort::SortPairs(temp, tb, run_b, sorted_b, iota, perm, (int)n, 0, bits_for(B), st));
  rule_out_kernel<<<grid, 256, 0, st>>>(perm, run_b, run_e, run_v, count, n, E, out_keys, out_vals, pos);
  MKG_LAUNCHED("rule_out_kernel");
  if (out_pos) {
    rule_entry_pos_kernel<<<grid, 256, 0, st>>>(scan, pos, n, out_pos);
    MKG_LAUNCHED("rule_entry_pos_kernel");
  }
  MKG_CUDA(cudaMemcpyAsync(count_out, count, sizeof(int64_t), cudaMemcpyDeviceToDevice, st));
  return MKG_OK;
}
