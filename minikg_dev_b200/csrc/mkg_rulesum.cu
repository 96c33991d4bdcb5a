// Sum (or max) over rules of a hop loop's final state without a full sort: sum_sp_3d
// (fastlog_bridge.py:17-23) and max_sp_3d (model_mmDRUM_kernel_sp.py:184-236) on a state in
// entity-major order (ascending entity, then row b * L + l), the order the key-slab engine
// emits.  There the L rules of one (entity, query) pair are adjacent, so each run of entries
// with one (e, b) folds in rule order, and only the runs need reordering, by query: for up to
// 1024 queries by the counting placement below (count pass, one scan, place pass); for more by
// the radix pipeline:
//  1. run heads: entry i starts a run when its (e, b) differs from entry i - 1's; an inclusive
//     scan numbers the runs (their (e, b) ascend entity-major);
//  2. each run head folds its run in rule order (fp32 sum, l ascending, as a sequential CPU
//     coalesce adds them; or the maximum) into run r = its number;
//  3. one stable radix pass over the runs' query b (the bits of B) puts them in (b, e) order;
//  4. the result keys b * E + e and values come out in that order, and every entry learns its
//     output position (the backward gathers the result's gradient through it).
// No host synchronisation: the run count stays on the device; the sort runs over all n slots,
// runs past the count carrying the query B - 1: the stable pass keeps them behind the real runs
// of that query (they come after every real run in the input), so the first count sorted
// entries are the real runs, and the pass needs only the bits of B - 1 (one 8-bit pass for up
// to 256 queries).
#include <cub/cub.cuh>

#include "mkg_common.cuh"

#define MKG_API extern "C" __attribute__((visibility("default")))

namespace mkg {
namespace {

size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

struct RuleSumLayout {
  size_t scan, run_b, run_e, run_v, sorted_b, iota, perm, pos, count, hist, temp, total;
  size_t temp_bytes;
};

int64_t rs_blocks(int64_t n);
constexpr int kRsMaxQueries = 1024;  // queries the counting placement takes (its shared histograms)

RuleSumLayout rule_sum_layout(int64_t n) {
  RuleSumLayout L{};
  size_t sort_b = 0, scan_b = 0, hscan_b = 0;
  const int64_t hist_items = (int64_t)kRsMaxQueries * rs_blocks(n) + 1;
  cub::DeviceRadixSort::SortPairs(nullptr, sort_b, (const int32_t*)nullptr, (int32_t*)nullptr,
                                  (const int32_t*)nullptr, (int32_t*)nullptr, (int)n);
  cub::DeviceScan::InclusiveSum(nullptr, scan_b, (int32_t*)nullptr, (int32_t*)nullptr, (int)n);
  cub::DeviceScan::ExclusiveSum(nullptr, hscan_b, (int32_t*)nullptr, (int32_t*)nullptr, (int)hist_items);
  L.temp_bytes = sort_b > scan_b ? sort_b : scan_b;
  if (hscan_b > L.temp_bytes) L.temp_bytes = hscan_b;
  size_t o = 0;
  L.scan = o; o += a256(4 * (size_t)n);      // run heads, then run numbers + 1
  L.run_b = o; o += a256(4 * (size_t)n);     // query of each run (B - 1 past the count)
  L.run_e = o; o += a256(8 * (size_t)n);     // entity of each run
  L.run_v = o; o += a256(4 * (size_t)n);     // value of each run
  L.sorted_b = o; o += a256(4 * (size_t)n);
  L.iota = o; o += a256(4 * (size_t)n);
  L.perm = o; o += a256(4 * (size_t)n);      // sorted position -> run
  L.pos = o; o += a256(4 * (size_t)n);       // run -> sorted position
  L.count = o; o += a256(8);
  L.hist = o; o += a256(4 * (size_t)hist_items);  // run heads per (query, block), then their scan
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
    run_b[i] = static_cast<int32_t>(B - 1);  // filler: overwritten for the runs that exist
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

// ---------------------------------------------------------------- counting placement
// For up to kRsMaxB queries the runs are placed by a stable counting sort over the query
// instead of the radix pass: a count pass histograms the run heads of each block by query, one
// scan of the histograms laid out query-major gives every (query, block) its first output
// position, and a place pass ranks each block's heads within their query (per-warp counts, then
// match_any in entry order), folds each run and writes it there.  Two reads of the keys, one
// of the values, the outputs and the per-entry positions; no sort of the entries.
constexpr int kRsThreads = 256;
constexpr int kRsWarps = kRsThreads / 32;
constexpr int kRsItems = 8;                                  // entries per lane
constexpr int64_t kRsWarpSpan = 32 * kRsItems;               // entries per warp
constexpr int64_t kRsTile = kRsWarps * kRsWarpSpan;          // entries per block
constexpr int kRsMaxB = kRsMaxQueries;

int64_t rs_blocks(int64_t n) { return (n + kRsTile - 1) / kRsTile; }

// (entity, query) of a valid key of the [B, L, E] space; false (and b = -1) otherwise
__device__ __forceinline__ bool decode_run(int64_t key, const FastDiv& E, int64_t L, int64_t B, int64_t& e,
                                           int32_t& b) {
  e = -1;
  b = -1;
  if (key < 0) return false;
  int64_t ee, bb;
  split_key(key, E, L, ee, bb);
  if (bb >= B) return false;
  e = ee;
  b = static_cast<int32_t>(bb);
  return true;
}

// A warp's entries: lane l holds entries wbase + u * 32 + l (u < kRsItems), so item u of the
// warp is 32 consecutive entries and the entry before lane l's is lane l - 1's (lane 31's of item
// u - 1 for lane 0).
struct RunItems {
  int64_t e[kRsItems];
  int32_t b[kRsItems];  // -1: invalid key, or past n
  unsigned head;        // bit u: entry u starts a run
};

__device__ __forceinline__ void load_runs(const int64_t* __restrict__ keys, int64_t n, const FastDiv& E, int64_t L,
                                          int64_t B, int64_t wbase, int lane, unsigned* err, RunItems& it) {
  int64_t ce = -1;  // lane 0: the entry before its next one
  int32_t cb = -1;
  if (lane == 0 && wbase > 0 && wbase - 1 < n) decode_run(keys[wbase - 1], E, L, B, ce, cb);
  it.head = 0;
#pragma unroll
  for (int u = 0; u < kRsItems; ++u) {
    const int64_t i = wbase + (int64_t)u * 32 + lane;
    int64_t e = -1;
    int32_t b = -1;
    const bool ok = i < n && decode_run(keys[i], E, L, B, e, b);
    if (i < n && !ok && err) raise_flag(err, MKG_DEV_BAD_KEY);
    int64_t pe = __shfl_up_sync(0xffffffffu, e, 1);
    int32_t pb = __shfl_up_sync(0xffffffffu, b, 1);
    if (lane == 0) { pe = ce; pb = cb; }
    ce = __shfl_sync(0xffffffffu, e, 31);
    cb = __shfl_sync(0xffffffffu, b, 31);
    const bool pok = pb >= 0;
    if (ok && (!pok || e != pe || b != pb)) it.head |= 1u << u;
    // not entity-major: runs of one (e, b) would split
    if (err && ok && pok && (e < pe || (e == pe && b < pb))) raise_flag(err, MKG_DEV_BAD_KEY);
    it.e[u] = e;
    it.b[u] = b;
  }
}

// bh[b * nblk + blk] = run heads of query b among block blk's entries
__global__ void __launch_bounds__(kRsThreads) rule_count_kernel(const int64_t* __restrict__ keys, int64_t n, FastDiv E,
                                                               int64_t L, int64_t B, int64_t nblk,
                                                               int32_t* __restrict__ bh, unsigned* err) {
  __shared__ int hist[kRsMaxB];
  for (int b = threadIdx.x; b < B; b += kRsThreads) hist[b] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  RunItems it;
  load_runs(keys, n, E, L, B, blockIdx.x * kRsTile + (int64_t)wid * kRsWarpSpan, lane, err, it);
#pragma unroll
  for (int u = 0; u < kRsItems; ++u)
    if ((it.head >> u) & 1u) atomicAdd(&hist[it.b[u]], 1);
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += kRsThreads) bh[(int64_t)b * nblk + blockIdx.x] = hist[b];
}

// bh_off: the exclusive scan of bh ([B * nblk + 1], the last entry the run count)
template <bool MAX>
__global__ void __launch_bounds__(kRsThreads) rule_place_kernel(
    const int64_t* __restrict__ keys, const float* __restrict__ vals, int64_t n, FastDiv E, int64_t L, int64_t B,
    int64_t nblk, const int32_t* __restrict__ bh_off, int64_t* __restrict__ out_keys, float* __restrict__ out_vals,
    int64_t* __restrict__ out_pos, int64_t* __restrict__ count) {
  __shared__ int base[kRsWarps][kRsMaxB];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (blockIdx.x == 0 && threadIdx.x == 0) *count = bh_off[B * nblk];
  for (int b = lane; b < B; b += 32) base[wid][b] = 0;
  const int64_t wbase = blockIdx.x * kRsTile + (int64_t)wid * kRsWarpSpan;
  RunItems it;
  load_runs(keys, n, E, L, B, wbase, lane, nullptr, it);
  __syncwarp();
#pragma unroll
  for (int u = 0; u < kRsItems; ++u)
    if ((it.head >> u) & 1u) atomicAdd(&base[wid][it.b[u]], 1);
  __syncthreads();
  // each warp's first position per query: the block's (from the scan), then the earlier warps'
  for (int b = threadIdx.x; b < B; b += kRsThreads) {
    int run = bh_off[(int64_t)b * nblk + blockIdx.x];
    for (int w = 0; w < kRsWarps; ++w) {
      const int t = base[w][b];
      base[w][b] = run;
      run += t;
    }
  }
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
#pragma unroll
  for (int u = 0; u < kRsItems; ++u) {
    const int64_t i = wbase + (int64_t)u * 32 + lane;
    const bool h = (it.head >> u) & 1u;
    const int32_t b = it.b[u];
    // heads of one query in this item: ranked by lane, after the warp's earlier ones
    const unsigned peers = __match_any_sync(0xffffffffu, h ? b : -1 - lane);
    const int pos = h ? base[wid][b] + __popc(peers & lt) : 0;
    __syncwarp();
    if (h && lane == 31 - __clz(peers)) base[wid][b] += __popc(peers);
    __syncwarp();
    // the run of a head: this entry and the following ones with the same (e, b), in rule order.
    // Within the item the following entries are the next lanes (up to the next head or invalid
    // entry): their values come by shuffle and are added one by one in lane order; a run that
    // reaches lane 31 continues from global memory.
    const float v = i < n ? vals[i] : 0.0f;
    const bool stop = h || b < 0;  // does not continue the run of the lane before
    float acc = v;
    bool open = h, tail = false;
    int len = 1;
    for (int k = 1; __ballot_sync(0xffffffffu, open) != 0u; ++k) {
      const float vk = __shfl_down_sync(0xffffffffu, v, k & 31);
      const bool sk = __shfl_down_sync(0xffffffffu, (int)stop, k & 31) != 0;
      if (open) {
        if (lane + k >= 32) {
          open = false;
          tail = true;
        } else if (sk) {
          open = false;
        } else {
          acc = MAX ? fmaxf(acc, vk) : __fadd_rn(acc, vk);
          ++len;
        }
      }
    }
    // each entry's result index: from the nearest head at or below its lane in this item (a
    // run begun in an earlier item is written by its head's global walk)
    const unsigned heads = __ballot_sync(0xffffffffu, h) & (0xffffffffu >> (31 - lane));
    const int src = heads ? 31 - __clz(heads) : lane;
    const int hpos = __shfl_sync(0xffffffffu, pos, src);
    if (out_pos && i < n) {
      if (b < 0) out_pos[i] = -1;  // an invalid key (flagged by the count pass)
      else if (heads) out_pos[i] = hpos;
    }
    if (h) {
      if (tail) {
        const int64_t e = it.e[u];
        for (int64_t j = i + len; j < n; ++j) {
          int64_t ej;
          int32_t bj;
          if (!decode_run(keys[j], E, L, B, ej, bj) || ej != e || bj != b) break;
          acc = MAX ? fmaxf(acc, vals[j]) : __fadd_rn(acc, vals[j]);
          if (out_pos) out_pos[j] = pos;
        }
      }
      out_keys[pos] = (int64_t)b * E.d + it.e[u];
      out_vals[pos] = acc;
    }
  }
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
  const FastDiv fe = FastDiv::of(E);
  if (B <= kRsMaxB) {  // counting placement
    const int64_t nblk = rs_blocks(n);
    auto* bh = reinterpret_cast<int32_t*>(w + Ly.hist);
    const int64_t items = B * nblk + 1;
    MKG_CUDA(cudaMemsetAsync(bh + items - 1, 0, sizeof(int32_t), st));
    rule_count_kernel<<<(unsigned)nblk, kRsThreads, 0, st>>>(keys, n, fe, L, B, nblk, bh, dev_err);
    MKG_LAUNCHED("rule_count_kernel");
    MKG_CUDA(cub::DeviceScan::ExclusiveSum(temp, tb, bh, bh, (int)items, st));
    if (mode == 1)
      rule_place_kernel<true><<<(unsigned)nblk, kRsThreads, 0, st>>>(keys, vals, n, fe, L, B, nblk, bh, out_keys,
                                                                     out_vals, out_pos, count_out);
    else
      rule_place_kernel<false><<<(unsigned)nblk, kRsThreads, 0, st>>>(keys, vals, n, fe, L, B, nblk, bh, out_keys,
                                                                      out_vals, out_pos, count_out);
    MKG_LAUNCHED("rule_place_kernel");
    return MKG_OK;
  }
  const int grid = grid_for(n, 256, persistent_blocks(8));
  rule_heads_kernel<<<grid, 256, 0, st>>>(keys, n, fe, L, B, scan, run_b, iota, dev_err);
  MKG_LAUNCHED("rule_heads_kernel");
  MKG_CUDA(cub::DeviceScan::InclusiveSum(temp, tb, scan, scan, (int)n, st));
  if (mode == 1)
    rule_runs_kernel<true><<<grid, 256, 0, st>>>(keys, vals, n, fe, L, B, scan, run_b, run_e, run_v, count);
  else
    rule_runs_kernel<false><<<grid, 256, 0, st>>>(keys, vals, n, fe, L, B, scan, run_b, run_e, run_v, count);
  MKG_LAUNCHED("rule_runs_kernel");
  // stable: runs of one query keep their ascending-entity order
  MKG_CUDA(cub::DeviceRadixSort::SortPairs(temp, tb, run_b, sorted_b, iota, perm, (int)n, 0, bits_for(B - 1), st));
  rule_out_kernel<<<grid, 256, 0, st>>>(perm, run_b, run_e, run_v, count, n, E, out_keys, out_vals, pos);
  MKG_LAUNCHED("rule_out_kernel");
  if (out_pos) {
    rule_entry_pos_kernel<<<grid, 256, 0, st>>>(scan, pos, n, out_pos);
    MKG_LAUNCHED("rule_entry_pos_kernel");
  }
  MKG_CUDA(cudaMemcpyAsync(count_out, count, sizeof(int64_t), cudaMemcpyDeviceToDevice, st));
  return MKG_OK;
}
