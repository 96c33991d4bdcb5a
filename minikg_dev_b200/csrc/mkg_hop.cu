// The per-hop op behind FastLogFunctionSparse3DTopK: degree-bucketed push expansion of a
// sparse [B, L, E] frontier over the ori / inv CSR with the exact 256-bucket edge cap,
// reduced on the fly (sum: fp32 atomics; max: packed 64-bit (value, fact id) atomicMax) into
// one of two key stores, then written as coalesced COO in key order:
//  * dense: slabs indexed by the output key (plus a hit byte per key for sums), compacted
//    by a tile scan -- for frontiers that touch a good share of the B x L x E key space;
//  * hash: open-addressing tables of 2^ceil(log2(2 * msg_bound)) slots (keys claimed with
//    atomicCAS, linear probing), radix-sorted by key -- when the message bound is far below
//    the key space (sparse frontiers on large graphs), so cost follows the messages.
// The backward walks the same messages and gathers the gradient from the same kind of store.
#include <algorithm>

#include <cub/cub.cuh>

#include "mkg_common.cuh"

namespace mkg {
namespace {

constexpr int kTailMax = 32;     // entries with <= 32 edges (both directions): thread per entry
constexpr int kHubMin = 4096;    // entries with  > 4096 edges: block per entry
constexpr int kHubThreads = 256;
constexpr int kMidWarps = 8;     // warps per block in the warp-per-entry kernel
constexpr int kTile = 4096;      // keys per compaction block (256 threads x 16)
constexpr int kTileThreads = 256;
constexpr int kHubStageMax = 4096;  // rule-weight rows up to this many channels are staged in smem
constexpr int64_t kHashRatio = 32;  // hash tables when 32 * msg_bound < key space
constexpr int64_t kMinSlots = 1024;
constexpr int64_t kMaxSlots = int64_t(1) << 30;  // CUB sorts take an int item count

size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

// Output entities: the destination range [lo, lo + extent) (the whole [0, E) by default).
int64_t range_lo(const mkg_hop_params& p) { return p.dst_hi > p.dst_lo ? p.dst_lo : 0; }
int64_t range_extent(const mkg_hop_params& p) { return p.dst_hi > p.dst_lo ? p.dst_hi - p.dst_lo : p.E; }

int64_t pow2_at_least(int64_t x) {
  int64_t c = kMinSlots;
  while (c < x) c <<= 1;
  return c;
}
int log2_exact(int64_t c) {
  int k = 0;
  while ((int64_t(1) << k) < c) ++k;
  return k;
}

struct HopLayout {
  bool hash;
  int bits;                // hash: keys < empty = 2^bits - 1 (radix sort over these bits)
  int64_t BLE, F, nblk;
  int64_t capm, capf;      // hash slots: ori / inv tables, ind table (and the entry map)
  // dense: per-slab strides in elements; every slab starts 256-byte aligned (the compaction
  // reads 16 hit bytes at a time as one uint4)
  int64_t sval, shit, spk;
  size_t off_val, off_hit, off_pk, off_lists, off_counts, off_blk, off_blkoff, off_cub, off_map, total;
  // hash: claimed keys, values (f32 / packed u64), their key-sorted copies, entry map values
  size_t off_tkey, off_tval, off_tpk, off_skey, off_sval, off_spk, off_mapkey;
  size_t off_gw64;         // backward: rule-weight gradient accumulated in fp64
  size_t off_gsp64;        // backward: frontier-entry gradient accumulated in fp64
  size_t cub_bytes;

  int64_t slots(int t) const { return t < 2 ? capm : capf; }
  int64_t base(int t) const { return t < 2 ? capm * t : 2 * capm; }
  unsigned long long empty() const { return (1ull << bits) - 1ull; }
};

bool use_hash(const mkg_hop_params& p) {
  if (p.accum == 1) return false;
  if (p.accum == 2) return true;
  const int64_t BLE = p.B * p.L * range_extent(p);
  return p.msg_bound > 0 && kHashRatio * p.msg_bound < BLE;
}

void hash_dims(HopLayout& L, const mkg_hop_params& p, int64_t F) {
  L.capm = pow2_at_least(2 * (p.msg_bound > 0 ? p.msg_bound : 1));
  L.capf = pow2_at_least(2 * (F > 0 ? F : 1));
  L.bits = 1;
  const int64_t key_space = std::max(L.BLE, p.B * p.L * p.E);  // the entry map uses full-range keys
  while (L.bits < 63 && (1ull << L.bits) - 1ull <= static_cast<unsigned long long>(key_space)) ++L.bits;
}

size_t scan_bytes(int64_t nblk) {
  size_t b = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, b, (int64_t*)nullptr, (int64_t*)nullptr, (int)(nblk + 1));
  return b;
}

template <class V>
size_t sort_bytes(int64_t n) {
  size_t b = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, b, (const unsigned long long*)nullptr, (unsigned long long*)nullptr,
                                  (const V*)nullptr, (V*)nullptr, (int)n);
  return b;
}

// Forward workspace.  Dense: value slabs (sum: ori, inv, ind; max: ind), hit slabs, packed
// slabs (max: ori, inv), per-tile counts and offsets.  Hash: three tables (ori, inv, ind)
// of claimed keys with f32 values (max: packed u64 for ori / inv) and their sorted copies.
// Both: the class lists.
HopLayout forward_layout(const mkg_hop_params& p, int64_t F) {
  HopLayout L{};
  L.BLE = p.B * p.L * range_extent(p);
  L.F = F;
  L.hash = use_hash(p);
  size_t o = 0;
  if (!L.hash) {
    L.nblk = (L.BLE + kTile - 1) / kTile;
    const int nval = p.agg_mode == 1 ? 1 : 3;
    L.sval = a256(4 * (size_t)L.BLE) / 4;
    L.shit = a256((size_t)L.BLE);
    L.spk = a256(8 * (size_t)L.BLE) / 8;
    L.off_val = o; o += 4 * (size_t)L.sval * nval;
    L.off_hit = o; o += (size_t)L.shit * nval;
    L.off_pk = o; o += p.agg_mode == 1 ? 8 * (size_t)L.spk * 2 : 0;
    L.off_blk = o; o += a256(8 * (size_t)(L.nblk + 1) * 3);
    L.off_blkoff = o; o += a256(8 * (size_t)(L.nblk + 1) * 3);
    L.cub_bytes = scan_bytes(L.nblk);
  } else {
    hash_dims(L, p, F);
    const size_t all = (size_t)(2 * L.capm + L.capf);
    L.off_tkey = o; o += a256(8 * all);
    L.off_tval = o; o += a256(4 * all);
    L.off_tpk = o; o += p.agg_mode == 1 ? a256(8 * (size_t)(2 * L.capm)) : 0;
    L.off_skey = o; o += a256(8 * all);
    L.off_sval = o; o += a256(4 * all);
    L.off_spk = o; o += p.agg_mode == 1 ? a256(8 * (size_t)(2 * L.capm)) : 0;
    L.cub_bytes = std::max(std::max(sort_bytes<float>(L.capm), sort_bytes<float>(L.capf)),
                           p.agg_mode == 1 ? sort_bytes<unsigned long long>(L.capm) : size_t(0));
  }
  L.off_lists = o; o += a256(4 * (size_t)(3 * F + 3));
  L.off_counts = o; o += a256(4 * 4);
  L.off_cub = o; o += a256(L.cub_bytes);
  L.off_map = 0;
  L.total = o;
  return L;
}

// Backward workspace: gradient stores (ori, inv, ind), class lists, the entry map (max).
HopLayout backward_layout(const mkg_hop_params& p, int64_t F) {
  HopLayout L{};
  L.BLE = p.B * p.L * range_extent(p);
  L.F = F;
  L.hash = use_hash(p);
  size_t o = 0;
  if (!L.hash) {
    L.sval = a256(4 * (size_t)L.BLE) / 4;
    L.off_val = o; o += 4 * (size_t)L.sval * 3;
    L.off_map = o; o += p.agg_mode == 1 ? a256(4 * (size_t)(p.B * p.L * p.E)) : 0;
  } else {
    hash_dims(L, p, F);
    const size_t all = (size_t)(2 * L.capm + L.capf);
    L.off_tkey = o; o += a256(8 * all);
    L.off_tval = o; o += a256(4 * all);
    L.off_mapkey = o; o += p.agg_mode == 1 ? a256(8 * (size_t)L.capf) : 0;
    L.off_map = o; o += p.agg_mode == 1 ? a256(4 * (size_t)L.capf) : 0;
  }
  L.off_lists = o; o += a256(4 * (size_t)(3 * F + 3));
  L.off_counts = o; o += a256(4 * 4);
  L.off_gw64 = o; o += a256(8 * (size_t)(p.B * p.L * p.n));
  L.off_gsp64 = o; o += a256(8 * (size_t)(F > 0 ? F : 1));
  L.total = o;
  return L;
}

struct Frontier {
  const int64_t* b;
  const int64_t* l;
  const int64_t* e;
  const float* v;
  int64_t F;
};

struct HopCtx {
  int64_t B, L, E, T, n, r_size, cap;
  int64_t lo, Eo;  // destination range [lo, lo + Eo); output keys are (b * L + l) * Eo + (dst - lo)
  int wot_i;
  DirCSR dir[2];
  EdgeFactor factor;
  const float* w;
  unsigned* err;
};

// ------------------------------------------------------------------ key stores
// Dense (keys == nullptr): the slot of a key is the key.  Hash: open addressing with linear
// probing over 2^k slots; a key claims its slot with atomicCAS from `empty`.  Probing is
// bounded by the table size; a full table sets MKG_DEV_TABLE_FULL and drops the message.
struct KeyTable {
  unsigned long long* keys;
  unsigned long long empty;
  int64_t mask;
  int shift;

  __device__ __forceinline__ int64_t home(unsigned long long key) const {
    return static_cast<int64_t>((key * 0x9E3779B97F4A7C15ull) >> shift);
  }
  __device__ __forceinline__ int64_t insert(unsigned long long key, unsigned* err) const {
    if (keys == nullptr) return static_cast<int64_t>(key);
    int64_t s = home(key);
    for (int64_t probe = 0; probe <= mask; ++probe) {
      unsigned long long cur = keys[s];
      if (cur == key) return s;
      if (cur == empty) {
        unsigned long long prev = atomicCAS(keys + s, empty, key);
        if (prev == empty || prev == key) return s;
      }
      s = (s + 1) & mask;
    }
    raise_flag(err, MKG_DEV_TABLE_FULL);
    return -1;
  }
  __device__ __forceinline__ int64_t find(unsigned long long key) const {
    if (keys == nullptr) return static_cast<int64_t>(key);
    int64_t s = home(key);
    for (int64_t probe = 0; probe <= mask; ++probe) {
      unsigned long long cur = keys[s];
      if (cur == key) return s;
      if (cur == empty) return -1;
      s = (s + 1) & mask;
    }
    return -1;
  }
};

KeyTable dense_table() { return KeyTable{nullptr, 0ull, 0, 64}; }
KeyTable hash_table(unsigned long long* keys, const HopLayout& L, int t) {
  const int64_t n = L.slots(t);
  return KeyTable{keys + L.base(t), L.empty(), n - 1, 64 - log2_exact(n)};
}

// ------------------------------------------------------------------ message sinks
// Each sink receives one message: direction d, output key, value inputs and fact id.
struct SumSink {
  float* val[2];
  uint8_t* hit[2];  // dense only
  KeyTable tab[2];
  unsigned* err;
  __device__ __forceinline__ void msg(int d, int64_t key, float v, int64_t /*fact*/) {
    const int64_t s = tab[d].insert(static_cast<unsigned long long>(key), err);
    if (s < 0) return;
    atomicAdd(val[d] + s, v);
    if (hit[d] != nullptr) hit[d][s] = 1;
  }
};

struct MaxSink {
  unsigned long long* pk[2];
  KeyTable tab[2];
  unsigned* err;
  __device__ __forceinline__ void msg(int d, int64_t key, float v, int64_t fact) {
    const int64_t s = tab[d].insert(static_cast<unsigned long long>(key), err);
    if (s < 0) return;
    atomicMax(pk[d] + s, pack_value_rank(v, static_cast<uint32_t>(fact)));
  }
};

// Output key of (b, l, dst) is out_key0 + dst; dst must lie in the destination range.
__device__ __forceinline__ int64_t out_key0(const HopCtx& c, int64_t b, int64_t l) { return (b * c.L + l) * c.Eo - c.lo; }
__device__ __forceinline__ bool in_range(const HopCtx& c, int64_t e) {
  return static_cast<uint64_t>(e - c.lo) < static_cast<uint64_t>(c.Eo);
}

// ------------------------------------------------------------------ entry classes
__device__ __forceinline__ bool load_entry(const Frontier& f, const HopCtx& c, int64_t i, int64_t& b,
                                           int64_t& l, int64_t& e) {
  b = f.b[i]; l = f.l[i]; e = f.e[i];
  if (b < 0 || b >= c.B || l < 0 || l >= c.L || e < 0 || e >= c.E) {
    raise_flag(c.err, MKG_DEV_BAD_ENTRY);
    return false;
  }
  return true;
}

// Sorts every frontier entry into tail / mid / hub lists (warp-aggregated appends) and
// emits its identity-channel message into the ind store (sum).
__global__ void classify_kernel(Frontier f, HopCtx c, int32_t* __restrict__ lists,
                                int32_t* __restrict__ counts, float* __restrict__ ind_val,
                                uint8_t* __restrict__ ind_hit, KeyTable ind_tab) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t base = warp0 * 32; base < f.F; base += nwarps * 32) {
    const int64_t i = base + lane;
    int cls = -1;
    if (i < f.F) {
      int64_t b, l, e;
      if (load_entry(f, c, i, b, l, e)) {
        if (ind_val != nullptr && in_range(c, e)) {
          const int64_t s = ind_tab.insert(static_cast<unsigned long long>(out_key0(c, b, l) + e), c.err);
          if (s >= 0) {
            float v = c.wot_i ? 0.0f : f.v[i] * c.w[(b * c.L + l) * c.n + (c.n - 1)];
            atomicAdd(ind_val + s, v);
            if (ind_hit != nullptr) ind_hit[s] = 1;
          }
        }
        int64_t d0 = c.dir[0].row_ptr[e + 1] - c.dir[0].row_ptr[e];
        int64_t d1 = c.dir[1].row_ptr[e + 1] - c.dir[1].row_ptr[e];
        int64_t tot = d0 + d1;
        bool capped = d0 > c.cap || d1 > c.cap;
        if (tot > 0) cls = (!capped && tot <= kTailMax) ? 0 : (tot <= kHubMin ? 1 : 2);
      }
    }
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      unsigned m = __ballot_sync(0xffffffffu, cls == k);
      if (m == 0) continue;
      int leader = __ffs(m) - 1;
      int pos0 = 0;
      if (lane == leader) pos0 = atomicAdd(counts + k, __popc(m));
      pos0 = __shfl_sync(0xffffffffu, pos0, leader);
      if (cls == k) lists[k * f.F + pos0 + __popc(m & ((1u << lane) - 1u))] = static_cast<int32_t>(i);
    }
  }
}

// Exact message counts: per entry min(out-degree, cap) per direction (cap <= 0: none).
__global__ void count_messages_kernel(Frontier f, HopCtx c, unsigned long long* __restrict__ out) {
  typedef cub::BlockReduce<long long, 256> Reduce;
  __shared__ typename Reduce::TempStorage tmp;
  long long m[2] = {0, 0};
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < f.F;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t b, l, e;
    if (!load_entry(f, c, i, b, l, e)) continue;
    for (int d = 0; d < 2; ++d) {
      const int64_t deg = c.dir[d].row_ptr[e + 1] - c.dir[d].row_ptr[e];
      m[d] += c.cap <= 0 ? 0 : (deg < c.cap ? deg : c.cap);
    }
  }
  for (int d = 0; d < 2; ++d) {
    long long t = Reduce(tmp).Sum(m[d]);
    if (threadIdx.x == 0 && t != 0) atomicAdd(out + d, static_cast<unsigned long long>(t));
    __syncthreads();
  }
}

// One message of direction d from CSR position p (shared by every traversal).
template <class Visit>
__device__ __forceinline__ void visit_position(const HopCtx& c, int d, int64_t p, const float* wrow,
                                               Visit& vis) {
  const DirCSR& cs = c.dir[d];
  int64_t dst = cs.col[p];
  int64_t fact = cs.order[p];
  int64_t ch = (d ? c.r_size : 0) + cs.rel[p];
  if (dst < 0 || dst >= c.E) { raise_flag(c.err, MKG_DEV_BAD_COL); return; }
  if (fact < 0 || fact >= c.T) { raise_flag(c.err, MKG_DEV_BAD_FACT); return; }
  if (ch < 0 || ch >= c.n - 1) { raise_flag(c.err, MKG_DEV_BAD_REL); return; }
  vis(d, dst, ch, wrow[ch], fact);
}

// Capped direction of one entry, executed by one full warp: 256-bucket histogram of the
// group weights (weighted by group sizes), threshold bucket + remain, then per group the
// take in group order, expanded cooperatively (fastlog.cu:2092-2112, 2167-2194, 2273-2322).
template <class Visit>
__device__ void warp_capped_direction(const HopCtx& c, int d, int64_t e, const float* wrow,
                                      int* hist, Visit& vis) {
  const int lane = threadIdx.x & 31;
  const DirCSR& cs = c.dir[d];
  const int64_t off = d ? c.r_size : 0;
  const int64_t g0 = cs.group_ptr[e], g1 = cs.group_ptr[e + 1];
  if (c.cap <= 0) return;  // every take is 0
  for (int k = lane; k < kNumBuckets; k += 32) hist[k] = 0;
  __syncwarp();
  for (int64_t g = g0 + lane; g < g1; g += 32) {
    int64_t ch = off + cs.group_rel[g];
    float wv = (ch >= 0 && ch < c.n - 1) ? wrow[ch] : 0.0f;
    atomicAdd(hist + weight_bucket(wv), cs.group_count[g]);
  }
  __syncwarp();
  // lane j owns buckets 255-8j .. 248-8j (descending)
  long long loc = 0;
#pragma unroll
  for (int t = 0; t < 8; ++t) loc += hist[255 - 8 * lane - t];
  long long incl = warp_inclusive_scan_ll(loc);
  unsigned hit = __ballot_sync(0xffffffffu, incl >= c.cap);
  int tb = 0;
  long long before = 0;
  if (hit != 0) {
    int jl = __ffs(hit) - 1;
    if (lane == jl) {
      long long cum = incl - loc;
      for (int t = 0; t < 8; ++t) {
        int bk = 255 - 8 * lane - t;
        long long cn = hist[bk];
        if (cum + cn >= c.cap) { tb = bk; before = cum; break; }
        cum += cn;
      }
    }
    tb = __shfl_sync(0xffffffffu, tb, jl);
    before = __shfl_sync(0xffffffffu, before, jl);
  }
  const long long remain = c.cap - before;
  __syncwarp();
  long long carry = 0;
  for (int64_t base = g0; base < g1; base += 32) {
    const int64_t g = base + lane;
    const bool valid = g < g1;
    int cnt = 0, bk = -1;
    int64_t st = 0, ch = 0;
    if (valid) {
      cnt = cs.group_count[g];
      st = cs.group_start[g];
      ch = off + cs.group_rel[g];
      bk = weight_bucket((ch >= 0 && ch < c.n - 1) ? wrow[ch] : 0.0f);
    }
    const long long x = (valid && bk == tb) ? cnt : 0;
    const long long xi = warp_inclusive_scan_ll(x);
    const long long prior = carry + xi - x;
    carry += __shfl_sync(0xffffffffu, xi, 31);
    int take = 0;
    if (valid) {
      if (bk > tb) take = cnt;
      else if (bk == tb) {
        long long t = remain - prior;
        take = static_cast<int>(t < 0 ? 0 : (t > cnt ? cnt : t));
      }
    }
    const int ti = warp_inclusive_scan(take);
    const int total = __shfl_sync(0xffffffffu, ti, 31);
    for (int kb = 0; kb < total; kb += 32) {
      const int k = kb + lane;
      // smallest lane j with ti[j] > k
      int lo = 0, hi = 31;
      while (lo < hi) {
        int mid = (lo + hi) >> 1;
        int v = __shfl_sync(0xffffffffu, ti, mid);
        if (v > k) hi = mid; else lo = mid + 1;
      }
      const int j = lo;
      const int tj_incl = __shfl_sync(0xffffffffu, ti, j);
      const int tj = __shfl_sync(0xffffffffu, take, j);
      const int64_t stj = __shfl_sync(0xffffffffu, st, j);
      if (k < total) visit_position(c, d, stj + (k - (tj_incl - tj)), wrow, vis);
    }
  }
}

// ---------------------------------------------------------------- forward visitors
template <class Sink>
struct FwdVisit {
  Sink sink;
  float sv;
  int64_t key0;
  const EdgeFactor* f;
  int64_t lo, Eo;
  __device__ __forceinline__ void operator()(int d, int64_t dst, int64_t /*ch*/, float wv, int64_t fact) {
    if (static_cast<uint64_t>(dst - lo) >= static_cast<uint64_t>(Eo)) return;  // another shard's destination
    float m = (*f)(fact);
    sink.msg(d, key0 + dst, (sv * wv) * m, fact);
  }
};

template <class Sink>
__global__ void push_tail_kernel(Frontier f, HopCtx c, const int32_t* __restrict__ list,
                                 const int32_t* __restrict__ count, Sink sink) {
  const int64_t n = *count;
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n;
       k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = list[k];
    int64_t b, l, e;
    if (!load_entry(f, c, i, b, l, e)) continue;
    const float* wrow = c.w + (b * c.L + l) * c.n;
    FwdVisit<Sink> vis{sink, f.v[i], out_key0(c, b, l), &c.factor, c.lo, c.Eo};
    for (int d = 0; d < 2; ++d) {
      const int64_t p0 = c.dir[d].row_ptr[e], p1 = c.dir[d].row_ptr[e + 1];
      for (int64_t p = p0; p < p1; ++p) visit_position(c, d, p, wrow, vis);
    }
  }
}

template <class Sink>
__global__ void __launch_bounds__(kMidWarps * 32) push_mid_kernel(Frontier f, HopCtx c,
                                                                  const int32_t* __restrict__ list,
                                                                  const int32_t* __restrict__ count,
                                                                  Sink sink) {
  __shared__ int hist_all[kMidWarps][kNumBuckets];
  int* hist = hist_all[threadIdx.x >> 5];
  const int lane = threadIdx.x & 31;
  const int64_t n = *count;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t k = warp0; k < n; k += nwarps) {
    const int64_t i = list[k];
    int64_t b, l, e;
    if (!load_entry(f, c, i, b, l, e)) continue;
    const float* wrow = c.w + (b * c.L + l) * c.n;
    FwdVisit<Sink> vis{sink, f.v[i], out_key0(c, b, l), &c.factor, c.lo, c.Eo};
    for (int d = 0; d < 2; ++d) {
      const int64_t p0 = c.dir[d].row_ptr[e], p1 = c.dir[d].row_ptr[e + 1];
      if (p1 - p0 <= c.cap) {
        for (int64_t p = p0 + lane; p < p1; p += 32) visit_position(c, d, p, wrow, vis);
      } else {
        warp_capped_direction(c, d, e, wrow, hist, vis);
      }
    }
  }
}

template <class Sink>
__global__ void __launch_bounds__(kHubThreads) push_hub_kernel(Frontier f, HopCtx c,
                                                               const int32_t* __restrict__ list,
                                                               const int32_t* __restrict__ count,
                                                               Sink sink) {
  __shared__ float wstage[kHubStageMax];
  __shared__ int hist[kNumBuckets];
  const int64_t n = *count;
  for (int64_t k = blockIdx.x; k < n; k += gridDim.x) {
    const int64_t i = list[k];
    int64_t b, l, e;
    if (!load_entry(f, c, i, b, l, e)) continue;
    const float* wg = c.w + (b * c.L + l) * c.n;
    const float* wrow = wg;
    if (c.n <= kHubStageMax) {  // stage the entry's rule-weight row in shared memory
      for (int t = threadIdx.x; t < c.n; t += blockDim.x) wstage[t] = wg[t];
      __syncthreads();
      wrow = wstage;
    }
    FwdVisit<Sink> vis{sink, f.v[i], out_key0(c, b, l), &c.factor, c.lo, c.Eo};
    for (int d = 0; d < 2; ++d) {
      const int64_t p0 = c.dir[d].row_ptr[e], p1 = c.dir[d].row_ptr[e + 1];
      if (p1 - p0 <= c.cap) {
        for (int64_t p = p0 + threadIdx.x; p < p1; p += blockDim.x) visit_position(c, d, p, wrow, vis);
      } else if (threadIdx.x < 32) {  // a capped direction emits at most cap messages: one warp
        warp_capped_direction(c, d, e, wrow, hist, vis);
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------- compaction
// flags: kind 0 = hit bytes, kind 1 = packed u64 != 0
__device__ __forceinline__ int tile_flags(int kind, const void* src, int64_t BLE, int64_t k0,
                                          unsigned& bits) {
  bits = 0;
  if (kind == 0) {
    const uint8_t* h = static_cast<const uint8_t*>(src);
    if (k0 + 16 <= BLE) {
      uint4 q = *reinterpret_cast<const uint4*>(h + k0);
      uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if ((w4[j >> 2] >> (8 * (j & 3))) & 0xffu) bits |= 1u << j;
    } else {
      for (int j = 0; j < 16 && k0 + j < BLE; ++j)
        if (h[k0 + j]) bits |= 1u << j;
    }
  } else {
    const unsigned long long* pk = static_cast<const unsigned long long*>(src);
    for (int j = 0; j < 16 && k0 + j < BLE; ++j)
      if (pk[k0 + j] != 0ull) bits |= 1u << j;
  }
  return __popc(bits);
}

__global__ void __launch_bounds__(kTileThreads) tile_count_kernel(int kind, const void* src, int64_t BLE,
                                                                  int64_t* __restrict__ blk_counts) {
  typedef cub::BlockReduce<int, kTileThreads> Reduce;
  __shared__ typename Reduce::TempStorage tmp;
  const int64_t k0 = blockIdx.x * (int64_t)kTile + threadIdx.x * 16;
  unsigned bits;
  int c = k0 < BLE ? tile_flags(kind, src, BLE, k0, bits) : 0;
  int tot = Reduce(tmp).Sum(c);
  if (threadIdx.x == 0) blk_counts[blockIdx.x] = tot;
}

__global__ void store_total_kernel(const int64_t* __restrict__ offs, int64_t nblk, int64_t* __restrict__ out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *out = offs[nblk];
}

__global__ void __launch_bounds__(kTileThreads) tile_emit_kernel(
    int kind, const void* src, const float* __restrict__ vals, int64_t BLE, int64_t L, int64_t E, int64_t lo,
    const int64_t* __restrict__ blk_off, int64_t count, int64_t* __restrict__ idx,
    float* __restrict__ out_val, int64_t* __restrict__ arg) {
  typedef cub::BlockScan<int, kTileThreads> Scan;
  __shared__ typename Scan::TempStorage tmp;
  const int64_t k0 = blockIdx.x * (int64_t)kTile + threadIdx.x * 16;
  unsigned bits = 0;
  int c = k0 < BLE ? tile_flags(kind, src, BLE, k0, bits) : 0;
  int excl;
  Scan(tmp).ExclusiveSum(c, excl);
  int64_t pos = blk_off[blockIdx.x] + excl;
  const unsigned long long* pk = static_cast<const unsigned long long*>(src);
  while (bits) {
    int j = __ffs(bits) - 1;
    bits &= bits - 1;
    int64_t key = k0 + j;
    if (pos < count) {
      int64_t be = key / (L * E), rem = key % (L * E);
      idx[pos] = be;
      idx[count + pos] = rem / E;
      idx[2 * count + pos] = rem % E + lo;
      if (kind == 0) {
        out_val[pos] = vals[key];
      } else {
        unsigned long long p = pk[key];
        out_val[pos] = packed_value(p);
        if (arg) arg[pos] = static_cast<int64_t>(packed_rank(p));
      }
    }
    ++pos;
  }
}

// ---------------------------------------------------------------- hash compaction
__global__ void fill_u64_kernel(unsigned long long* __restrict__ p, int64_t n, unsigned long long v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

// Claimed slots of a key-sorted table = position of the first empty key (empties sort last).
__global__ void count_claimed_kernel(const unsigned long long* __restrict__ sorted, int64_t n,
                                     unsigned long long empty, int64_t* __restrict__ out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (sorted[mid] < empty) lo = mid + 1; else hi = mid;
  }
  *out = lo;
}

__global__ void hash_emit_kernel(const unsigned long long* __restrict__ skey, const float* __restrict__ sval,
                                 const unsigned long long* __restrict__ spk, int64_t count, int64_t L, int64_t Eo,
                                 int64_t lo, int64_t* __restrict__ idx, float* __restrict__ out_val,
                                 int64_t* __restrict__ arg) {
  for (int64_t pos = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; pos < count;
       pos += (int64_t)gridDim.x * blockDim.x) {
    const int64_t key = static_cast<int64_t>(skey[pos]);
    const int64_t be = key / (L * Eo), rem = key % (L * Eo);
    idx[pos] = be;
    idx[count + pos] = rem / Eo;
    idx[2 * count + pos] = rem % Eo + lo;
    if (spk != nullptr) {
      const unsigned long long p = spk[pos];
      out_val[pos] = packed_value(p);
      if (arg) arg[pos] = static_cast<int64_t>(packed_rank(p));
    } else {
      out_val[pos] = sval[pos];
    }
  }
}

// ---------------------------------------------------------------- backward
// Gradient store of one hop: values per output key of ori / inv (dense slab or hash table).
struct GradStore {
  const float* val[2];
  KeyTable tab[2];
};

// Incoming gradient keys must lie in the destination range (the forward produced no others).
__global__ void scatter_grad_kernel(mkg_coo3 g, int64_t B, int64_t L, int64_t lo, int64_t Eo, KeyTable tab,
                                    float* __restrict__ vals, unsigned* err) {
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < g.nnz;
       k += (int64_t)gridDim.x * blockDim.x) {
    int64_t b = g.indices[k], l = g.indices[g.nnz + k], e = g.indices[2 * g.nnz + k] - lo;
    if (b < 0 || b >= B || l < 0 || l >= L || e < 0 || e >= Eo) { raise_flag(err, MKG_DEV_BAD_KEY); continue; }
    const int64_t s = tab.insert(static_cast<unsigned long long>((b * L + l) * Eo + e), err);
    if (s >= 0) atomicAdd(vals + s, g.values[k]);
  }
}

// Identity channel: grad_sp[i] = g_ind(key_i) * w[b,l,n-1] (initialises grad_sp) and
// grad_w[b,l,n-1] += g_ind * sv (fastlog.cu:2608-2644); also fills the key -> entry map
// (full-range keys) used by the argmax backward.  The entry and rule-weight gradients are fp64
// sums of fp64 products (rounded once at the end): both are sums whose terms cancel, where
// fp32-rounded terms drifted past 1e-5 of the result.
__global__ void backward_entry_init_kernel(Frontier f, HopCtx c, KeyTable ind_tab, const float* __restrict__ g_ind,
                                           double* __restrict__ grad_sp, double* __restrict__ grad_w,
                                           KeyTable map_tab, int32_t* __restrict__ entry_map) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < f.F;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t b, l, e;
    if (!load_entry(f, c, i, b, l, e)) { grad_sp[i] = 0.0; continue; }
    if (entry_map) {
      const int64_t s = map_tab.insert(static_cast<unsigned long long>((b * c.L + l) * c.E + e), c.err);
      if (s >= 0) entry_map[s] = static_cast<int32_t>(i);
    }
    double gsp = 0.0;
    if (!c.wot_i && in_range(c, e)) {
      const int64_t wi = (b * c.L + l) * c.n + (c.n - 1);
      const int64_t s = ind_tab.find(static_cast<unsigned long long>(out_key0(c, b, l) + e));
      float g = s >= 0 ? g_ind[s] : 0.0f;
      if (g != 0.0f) {
        gsp = (double)g * (double)c.w[wi];
        atomicAdd(grad_w + wi, (double)g * (double)f.v[i]);
      }
    }
    grad_sp[i] = gsp;
  }
}

__device__ __forceinline__ float edge_grad_factor(const EdgeFactor& f, int64_t fact) {
  if (f.weight == nullptr) return 0.0f;
  float ew = f.weight[fact];
  if (f.is_score) return 1.0f / fmaxf(ew, 1e-12f);
  float z = -ew * f.scale;
  float s = static_cast<float>(1.0 / (1.0 + exp(static_cast<double>(z))));
  return f.scale * (1.0f - s);
}

// Sum backward per message: g at the output key, grad_sp += (g*m)*w (accumulated per
// entry), grad_w += (g*m)*sv, grad_edge[fact] += (((g*sv)*w)*m)*factor.
struct BwdVisit {
  GradStore gs;
  double* grad_w;  // fp64 accumulator: every fp32 product added exactly, rounded once
  float* grad_edge;
  const EdgeFactor* f;
  float sv;
  int64_t key0, wbase;
  double acc;  // the entry's gradient (fp64 products, fp64 sum)
  int64_t lo, Eo;
  __device__ __forceinline__ void operator()(int d, int64_t dst, int64_t ch, float wv, int64_t fact) {
    if (static_cast<uint64_t>(dst - lo) >= static_cast<uint64_t>(Eo)) return;  // another shard's destination
    const int64_t s = gs.tab[d].find(static_cast<unsigned long long>(key0 + dst));
    if (s < 0) return;
    float g = gs.val[d][s];
    if (g == 0.0f) return;
    float m = (*f)(fact);
    const double gm = (double)g * (double)m;
    acc += gm * (double)wv;
    atomicAdd(grad_w + wbase + ch, gm * (double)sv);
    if (grad_edge) atomicAdd(grad_edge + fact, (((g * sv) * wv) * m) * edge_grad_factor(*f, fact));
  }
};

__global__ void bwd_tail_kernel(Frontier f, HopCtx c, const int32_t* __restrict__ list,
                                const int32_t* __restrict__ count, GradStore gs, double* __restrict__ grad_sp,
                                double* __restrict__ grad_w, float* __restrict__ grad_edge) {
  const int64_t n = *count;
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n;
       k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = list[k];
    int64_t b, l, e;
    if (!load_entry(f, c, i, b, l, e)) continue;
    const float* wrow = c.w + (b * c.L + l) * c.n;
    BwdVisit vis{gs, grad_w, grad_edge, &c.factor, f.v[i], out_key0(c, b, l), (b * c.L + l) * c.n, 0.0f, c.lo, c.Eo};
    for (int d = 0; d < 2; ++d) {
      const int64_t p0 = c.dir[d].row_ptr[e], p1 = c.dir[d].row_ptr[e + 1];
      for (int64_t p = p0; p < p1; ++p) visit_position(c, d, p, wrow, vis);
    }
    grad_sp[i] += vis.acc;
  }
}

__global__ void __launch_bounds__(kMidWarps * 32) bwd_mid_kernel(
    Frontier f, HopCtx c, const int32_t* __restrict__ list, const int32_t* __restrict__ count, GradStore gs,
    double* __restrict__ grad_sp, double* __restrict__ grad_w, float* __restrict__ grad_edge) {
  __shared__ int hist_all[kMidWarps][kNumBuckets];
  int* hist = hist_all[threadIdx.x >> 5];
  const int lane = threadIdx.x & 31;
  const int64_t n = *count;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t k = warp0; k < n; k += nwarps) {
    const int64_t i = list[k];
    int64_t b, l, e;
    if (!load_entry(f, c, i, b, l, e)) continue;
    const float* wrow = c.w + (b * c.L + l) * c.n;
    BwdVisit vis{gs, grad_w, grad_edge, &c.factor, f.v[i], out_key0(c, b, l), (b * c.L + l) * c.n, 0.0f, c.lo, c.Eo};
    for (int d = 0; d < 2; ++d) {
      const int64_t p0 = c.dir[d].row_ptr[e], p1 = c.dir[d].row_ptr[e + 1];
      if (p1 - p0 <= c.cap) {
        for (int64_t p = p0 + lane; p < p1; p += 32) visit_position(c, d, p, wrow, vis);
      } else {
        warp_capped_direction(c, d, e, wrow, hist, vis);
      }
    }
    const double tot = warp_sum_f64(vis.acc);
    if (lane == 0) grad_sp[i] += tot;
  }
}

__global__ void __launch_bounds__(kHubThreads) bwd_hub_kernel(
    Frontier f, HopCtx c, const int32_t* __restrict__ list, const int32_t* __restrict__ count, GradStore gs,
    double* __restrict__ grad_sp, double* __restrict__ grad_w, float* __restrict__ grad_edge) {
  __shared__ float wstage[kHubStageMax];
  __shared__ int hist[kNumBuckets];
  __shared__ double part[kHubThreads / 32];
  const int64_t n = *count;
  for (int64_t k = blockIdx.x; k < n; k += gridDim.x) {
    const int64_t i = list[k];
    int64_t b, l, e;
    if (!load_entry(f, c, i, b, l, e)) continue;
    const float* wg = c.w + (b * c.L + l) * c.n;
    const float* wrow = wg;
    if (c.n <= kHubStageMax) {
      for (int t = threadIdx.x; t < c.n; t += blockDim.x) wstage[t] = wg[t];
      __syncthreads();
      wrow = wstage;
    }
    BwdVisit vis{gs, grad_w, grad_edge, &c.factor, f.v[i], out_key0(c, b, l), (b * c.L + l) * c.n, 0.0f, c.lo, c.Eo};
    for (int d = 0; d < 2; ++d) {
      const int64_t p0 = c.dir[d].row_ptr[e], p1 = c.dir[d].row_ptr[e + 1];
      if (p1 - p0 <= c.cap) {
        for (int64_t p = p0 + threadIdx.x; p < p1; p += blockDim.x) visit_position(c, d, p, wrow, vis);
      } else if (threadIdx.x < 32) {
        warp_capped_direction(c, d, e, wrow, hist, vis);
      }
    }
    const double ws = warp_sum_f64(vis.acc);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ws;
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0.0;
      for (int q = 0; q < kHubThreads / 32; ++q) t += part[q];
      grad_sp[i] += t;
    }
    __syncthreads();
  }
}

// Max backward (full destination range): the gradient of every output key goes to its
// argmax message only (fastlog_kernel.py:153-167 + fastlog.cu:2646-2676).
__global__ void bwd_argmax_kernel(int d, mkg_coo3 out, const int64_t* __restrict__ arg, Frontier f, HopCtx c,
                                  KeyTable gtab, const float* __restrict__ gvals, KeyTable map_tab,
                                  const int32_t* __restrict__ entry_map, const int32_t* __restrict__ fhead,
                                  const int32_t* __restrict__ ftail, const int16_t* __restrict__ frel,
                                  double* __restrict__ grad_sp, double* __restrict__ grad_w,
                                  float* __restrict__ grad_edge) {
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < out.nnz;
       k += (int64_t)gridDim.x * blockDim.x) {
    int64_t b = out.indices[k], l = out.indices[out.nnz + k], dst = out.indices[2 * out.nnz + k];
    if (b < 0 || b >= c.B || l < 0 || l >= c.L || dst < 0 || dst >= c.E) { raise_flag(c.err, MKG_DEV_BAD_KEY); continue; }
    const int64_t gs = gtab.find(static_cast<unsigned long long>((b * c.L + l) * c.E + dst));
    float g = gs >= 0 ? gvals[gs] : 0.0f;
    if (g == 0.0f) continue;
    int64_t fact = arg[k];
    if (fact < 0 || fact >= c.T) { raise_flag(c.err, MKG_DEV_BAD_FACT); continue; }
    int64_t src = d ? ftail[fact] : fhead[fact];
    int64_t ch = (d ? c.r_size : 0) + frel[fact];
    if (src < 0 || src >= c.E || ch < 0 || ch >= c.n - 1) { raise_flag(c.err, MKG_DEV_BAD_COL); continue; }
    const int64_t ms = map_tab.find(static_cast<unsigned long long>((b * c.L + l) * c.E + src));
    int32_t i = ms >= 0 ? entry_map[ms] : -1;
    if (i < 0 || i >= f.F) { raise_flag(c.err, MKG_DEV_BAD_ENTRY); continue; }
    float m = c.factor(fact);
    float sv = f.v[i];
    int64_t wi = (b * c.L + l) * c.n + ch;
    float wv = c.w[wi];
    const double gm = (double)g * (double)m;
    atomicAdd(grad_sp + i, gm * (double)wv);
    atomicAdd(grad_w + wi, gm * (double)sv);
    if (grad_edge) atomicAdd(grad_edge + fact, (((g * sv) * wv) * m) * edge_grad_factor(c.factor, fact));
  }
}

HopCtx make_ctx(const mkg_graph* g, const float* w, const mkg_edge_factor* ef, const mkg_hop_params* p,
                unsigned* err) {
  HopCtx c;
  c.B = p->B; c.L = p->L; c.E = p->E; c.T = g->num_facts; c.n = p->n; c.r_size = p->r_size;
  c.cap = p->topk_edges; c.wot_i = p->wot_i;
  c.lo = range_lo(*p); c.Eo = range_extent(*p);
  c.dir[0] = make_dir(g->ori);
  c.dir[1] = make_dir(g->inv);
  c.factor = make_factor(*ef);
  c.w = w;
  c.err = err;
  return c;
}

int check_hop_args(const mkg_graph* g, const mkg_frontier* f, const float* w, const mkg_edge_factor* ef,
                   const mkg_hop_params* p) {
  MKG_REQUIRE(g && f && w && ef && p, "hop: null argument");
  MKG_REQUIRE(p->B >= 1 && p->L >= 1 && p->E >= 1 && p->n >= 1, "hop: B, L, E, n must be positive");
  MKG_REQUIRE(p->E == g->num_entities, "hop: E=%lld does not match the graph (%lld entities)",
              (long long)p->E, (long long)g->num_entities);
  MKG_REQUIRE(p->agg_mode == 0 || p->agg_mode == 1, "hop: agg_mode must be 0 or 1");
  MKG_REQUIRE(f->nnz >= 0 && f->nnz < (int64_t(1) << 31), "hop: frontier size out of range");
  MKG_REQUIRE(p->r_size >= 0, "hop: r_size must be non-negative");
  MKG_REQUIRE(g->num_facts < (int64_t(1) << 31) - 1, "hop: too many facts for 32-bit argmax ranks");
  MKG_REQUIRE(p->dst_hi <= p->dst_lo || (p->dst_lo >= 0 && p->dst_hi <= p->E),
              "hop: destination range [%lld, %lld) outside [0, E=%lld)", (long long)p->dst_lo,
              (long long)p->dst_hi, (long long)p->E);
  MKG_REQUIRE(p->msg_bound >= 0 && p->msg_bound < (int64_t(1) << 40), "hop: msg_bound out of range");
  MKG_REQUIRE(p->accum >= 0 && p->accum <= 2, "hop: accum must be 0, 1 or 2");
  MKG_REQUIRE(p->merge_outputs == 0 || (p->merge_outputs == 1 && p->agg_mode == 0),
              "hop: merge_outputs needs agg_mode 0");
  MKG_REQUIRE(p->B * p->L * p->E < (int64_t(1) << 62), "hop: key space B*L*E too large");
  return MKG_OK;
}

}  // namespace

int hop_count_messages(const mkg_graph* g, const mkg_frontier* fr, const mkg_hop_params* p, int64_t* counts_out,
                       unsigned* err, cudaStream_t st) {
  MKG_REQUIRE(g && fr && p && counts_out, "hop_count_messages: null argument");
  MKG_REQUIRE(p->B >= 1 && p->L >= 1 && p->E == g->num_entities, "hop_count_messages: bad shape");
  MKG_REQUIRE(fr->nnz >= 0, "hop_count_messages: negative frontier size");
  MKG_CUDA(cudaMemsetAsync(counts_out, 0, 2 * sizeof(int64_t), st));
  if (fr->nnz == 0) return MKG_OK;
  HopCtx c{};
  c.B = p->B; c.L = p->L; c.E = p->E; c.cap = p->topk_edges; c.err = err;
  c.dir[0] = make_dir(g->ori);
  c.dir[1] = make_dir(g->inv);
  Frontier f{fr->batch, fr->level, fr->entity, fr->value, fr->nnz};
  count_messages_kernel<<<grid_for(fr->nnz, 256, persistent_blocks(4)), 256, 0, st>>>(
      f, c, reinterpret_cast<unsigned long long*>(counts_out));
  MKG_LAUNCHED("count_messages_kernel");
  return MKG_OK;
}

size_t hop_forward_workspace_bytes(const mkg_hop_params* p, int64_t nnz) {
  return forward_layout(*p, nnz).total + 256;
}

int hop_forward(const mkg_graph* g, const mkg_frontier* fr, const float* w, const mkg_edge_factor* ef,
                const mkg_hop_params* p, void* ws, size_t ws_bytes, int64_t* counts_out, unsigned* err,
                cudaStream_t st) {
  int rc = check_hop_args(g, fr, w, ef, p);
  if (rc) return rc;
  MKG_REQUIRE(counts_out, "hop_forward: counts_out is null");
  HopLayout lay = forward_layout(*p, fr->nnz);
  if (lay.hash && (lay.capm > kMaxSlots || lay.capf > kMaxSlots)) {
    set_error("hop_forward: %lld messages per direction exceed one hash table (2^30 slots); split the batch",
              (long long)p->msg_bound);
    return MKG_ERR_CAPACITY;
  }
  MKG_REQUIRE(ws && ws_bytes >= lay.total, "hop_forward: workspace too small (%zu < %zu)", ws_bytes, lay.total);
  char* base = static_cast<char*>(ws);
  const int64_t BLE = lay.BLE, F = fr->nnz;
  int32_t* lists = reinterpret_cast<int32_t*>(base + lay.off_lists);
  int32_t* counts = reinterpret_cast<int32_t*>(base + lay.off_counts);
  void* cubtmp = base + lay.off_cub;
  MKG_CUDA(cudaMemsetAsync(counts, 0, 16, st));
  HopCtx c = make_ctx(g, w, ef, p, err);
  Frontier f{fr->batch, fr->level, fr->entity, fr->value, F};
  const int tb = persistent_blocks(8), mb = persistent_blocks(4), hb = persistent_blocks(2);

  if (!lay.hash) {
    float* val = reinterpret_cast<float*>(base + lay.off_val);
    uint8_t* hit = reinterpret_cast<uint8_t*>(base + lay.off_hit);
    unsigned long long* pk = reinterpret_cast<unsigned long long*>(base + lay.off_pk);
    int64_t* blk = reinterpret_cast<int64_t*>(base + lay.off_blk);
    int64_t* blkoff = reinterpret_cast<int64_t*>(base + lay.off_blkoff);
    const int nval = p->agg_mode == 1 ? 1 : 3;
    const int64_t SV = lay.sval, SH = lay.shit, SP = lay.spk;
    MKG_CUDA(cudaMemsetAsync(val, 0, 4 * (size_t)SV * nval, st));
    MKG_CUDA(cudaMemsetAsync(hit, 0, (size_t)SH * nval, st));
    if (p->agg_mode == 1) MKG_CUDA(cudaMemsetAsync(pk, 0, 8 * (size_t)SP * 2, st));
    // ind slab: the last value slab (index 2 for sum, 0 for max); merged: all into slab 0
    const bool merge = p->merge_outputs != 0;
    float* ind_val = merge ? val : val + SV * (nval - 1);
    uint8_t* ind_hit = merge ? hit : hit + SH * (nval - 1);
    const KeyTable dn = dense_table();
    if (F > 0) {
      classify_kernel<<<grid_for(F, 256, persistent_blocks(8)), 256, 0, st>>>(f, c, lists, counts, ind_val, ind_hit, dn);
      MKG_LAUNCHED("classify_kernel");
      if (p->agg_mode == 0) {
        SumSink s{{val, merge ? val : val + SV}, {hit, merge ? hit : hit + SH}, {dn, dn}, err};
        push_tail_kernel<SumSink><<<tb, 256, 0, st>>>(f, c, lists, counts, s);
        push_mid_kernel<SumSink><<<mb, kMidWarps * 32, 0, st>>>(f, c, lists + F, counts + 1, s);
        push_hub_kernel<SumSink><<<hb, kHubThreads, 0, st>>>(f, c, lists + 2 * F, counts + 2, s);
      } else {
        MaxSink s{{pk, pk + SP}, {dn, dn}, err};
        push_tail_kernel<MaxSink><<<tb, 256, 0, st>>>(f, c, lists, counts, s);
        push_mid_kernel<MaxSink><<<mb, kMidWarps * 32, 0, st>>>(f, c, lists + F, counts + 1, s);
        push_hub_kernel<MaxSink><<<hb, kHubThreads, 0, st>>>(f, c, lists + 2 * F, counts + 2, s);
      }
      MKG_LAUNCHED("push kernels");
    }
    // per-tile counts and offsets of the three outputs (merged: output 0 only)
    if (merge) MKG_CUDA(cudaMemsetAsync(counts_out + 1, 0, 2 * sizeof(int64_t), st));
    for (int which = 0; which < (merge ? 1 : 3); ++which) {
      int kind;
      const void* src;
      if (p->agg_mode == 1 && which < 2) { kind = 1; src = pk + SP * which; }
      else { kind = 0; src = hit + SH * (p->agg_mode == 1 ? 0 : which); }
      int64_t* bc = blk + (lay.nblk + 1) * which;
      int64_t* bo = blkoff + (lay.nblk + 1) * which;
      MKG_CUDA(cudaMemsetAsync(bc + lay.nblk, 0, 8, st));
      tile_count_kernel<<<(unsigned)lay.nblk, kTileThreads, 0, st>>>(kind, src, BLE, bc);
      MKG_LAUNCHED("tile_count_kernel");
      size_t b = lay.cub_bytes;
      MKG_CUDA(cub::DeviceScan::ExclusiveSum(cubtmp, b, bc, bo, (int)(lay.nblk + 1), st));
      store_total_kernel<<<1, 32, 0, st>>>(bo, lay.nblk, counts_out + which);
      MKG_LAUNCHED("store_total_kernel");
    }
    return MKG_OK;
  }

  // hash tables
  unsigned long long* tkey = reinterpret_cast<unsigned long long*>(base + lay.off_tkey);
  float* tval = reinterpret_cast<float*>(base + lay.off_tval);
  unsigned long long* tpk = reinterpret_cast<unsigned long long*>(base + lay.off_tpk);
  unsigned long long* skey = reinterpret_cast<unsigned long long*>(base + lay.off_skey);
  float* sval = reinterpret_cast<float*>(base + lay.off_sval);
  unsigned long long* spk = reinterpret_cast<unsigned long long*>(base + lay.off_spk);
  const int64_t all = 2 * lay.capm + lay.capf;
  fill_u64_kernel<<<grid_for(all, 256, persistent_blocks(8)), 256, 0, st>>>(tkey, all, lay.empty());
  MKG_LAUNCHED("fill_u64_kernel");
  MKG_CUDA(cudaMemsetAsync(tval, 0, 4 * (size_t)all, st));
  if (p->agg_mode == 1) MKG_CUDA(cudaMemsetAsync(tpk, 0, 8 * (size_t)(2 * lay.capm), st));
  const bool merge = p->merge_outputs != 0;
  const KeyTable t0 = hash_table(tkey, lay, 0);
  const KeyTable t1 = merge ? t0 : hash_table(tkey, lay, 1), t2 = merge ? t0 : hash_table(tkey, lay, 2);
  if (F > 0) {
    classify_kernel<<<grid_for(F, 256, persistent_blocks(8)), 256, 0, st>>>(
        f, c, lists, counts, tval + lay.base(merge ? 0 : 2), nullptr, t2);
    MKG_LAUNCHED("classify_kernel");
    if (p->agg_mode == 0) {
      SumSink s{{tval + lay.base(0), tval + lay.base(merge ? 0 : 1)}, {nullptr, nullptr}, {t0, t1}, err};
      push_tail_kernel<SumSink><<<tb, 256, 0, st>>>(f, c, lists, counts, s);
      push_mid_kernel<SumSink><<<mb, kMidWarps * 32, 0, st>>>(f, c, lists + F, counts + 1, s);
      push_hub_kernel<SumSink><<<hb, kHubThreads, 0, st>>>(f, c, lists + 2 * F, counts + 2, s);
    } else {
      MaxSink s{{tpk + lay.base(0), tpk + lay.base(1)}, {t0, t1}, err};
      push_tail_kernel<MaxSink><<<tb, 256, 0, st>>>(f, c, lists, counts, s);
      push_mid_kernel<MaxSink><<<mb, kMidWarps * 32, 0, st>>>(f, c, lists + F, counts + 1, s);
      push_hub_kernel<MaxSink><<<hb, kHubThreads, 0, st>>>(f, c, lists + 2 * F, counts + 2, s);
    }
    MKG_LAUNCHED("push kernels");
  }
  if (merge) MKG_CUDA(cudaMemsetAsync(counts_out + 1, 0, 2 * sizeof(int64_t), st));
  for (int t = 0; t < (merge ? 1 : 3); ++t) {
    const int64_t n = lay.slots(t), o = lay.base(t);
    size_t b = lay.cub_bytes;
    if (p->agg_mode == 1 && t < 2) {
      MKG_CUDA(cub::DeviceRadixSort::SortPairs(cubtmp, b, tkey + o, skey + o, tpk + o, spk + o, (int)n, 0,
                                               lay.bits, st));
    } else {
      MKG_CUDA(cub::DeviceRadixSort::SortPairs(cubtmp, b, tkey + o, skey + o, tval + o, sval + o, (int)n, 0,
                                               lay.bits, st));
    }
    count_claimed_kernel<<<1, 32, 0, st>>>(skey + o, n, lay.empty(), counts_out + t);
    MKG_LAUNCHED("count_claimed_kernel");
  }
  return MKG_OK;
}

int hop_emit(const mkg_hop_params* p, int64_t nnz, const void* ws, size_t ws_bytes, int which,
                   int64_t count, int64_t* indices, float* values, int64_t* arg, cudaStream_t st) {
  MKG_REQUIRE(p && ws, "hop_emit: null argument");
  MKG_REQUIRE(which >= 0 && which < 3, "hop_emit: which must be 0, 1 or 2");
  HopLayout lay = forward_layout(*p, nnz);
  MKG_REQUIRE(ws_bytes >= lay.total, "hop_emit: workspace too small");
  if (count == 0) return MKG_OK;
  MKG_REQUIRE(indices && values, "hop_emit: null output");
  const char* base = static_cast<const char*>(ws);
  if (lay.hash) {
    MKG_REQUIRE(count <= lay.slots(which), "hop_emit: count exceeds the table");
    const int64_t o = lay.base(which);
    const unsigned long long* skey = reinterpret_cast<const unsigned long long*>(base + lay.off_skey) + o;
    const float* sval = reinterpret_cast<const float*>(base + lay.off_sval) + o;
    const unsigned long long* spk =
        (p->agg_mode == 1 && which < 2) ? reinterpret_cast<const unsigned long long*>(base + lay.off_spk) + o : nullptr;
    hash_emit_kernel<<<grid_for(count, 256, persistent_blocks(8)), 256, 0, st>>>(
        skey, sval, spk, count, p->L, range_extent(*p), range_lo(*p), indices, values, spk ? arg : nullptr);
    MKG_LAUNCHED("hash_emit_kernel");
    return MKG_OK;
  }
  const int64_t BLE = lay.BLE;
  const float* val = reinterpret_cast<const float*>(base + lay.off_val);
  const uint8_t* hit = reinterpret_cast<const uint8_t*>(base + lay.off_hit);
  const unsigned long long* pk = reinterpret_cast<const unsigned long long*>(base + lay.off_pk);
  const int64_t* blkoff = reinterpret_cast<const int64_t*>(base + lay.off_blkoff) + (lay.nblk + 1) * which;
  int kind;
  const void* src;
  const float* vals = nullptr;
  if (p->agg_mode == 1 && which < 2) { kind = 1; src = pk + lay.spk * which; }
  else {
    int slot = p->agg_mode == 1 ? 0 : which;
    kind = 0; src = hit + lay.shit * slot; vals = val + lay.sval * slot;
  }
  tile_emit_kernel<<<(unsigned)lay.nblk, kTileThreads, 0, st>>>(kind, src, vals, BLE, p->L, range_extent(*p),
                                                               range_lo(*p), blkoff, count, indices, values,
                                                               kind == 1 ? arg : nullptr);
  MKG_LAUNCHED("tile_emit_kernel");
  return MKG_OK;
}

namespace {
__global__ void round_gw_kernel(const double* __restrict__ gw64, int64_t count, float* __restrict__ grad_w) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
    grad_w[i] = static_cast<float>(gw64[i]);
}
}  // namespace

size_t hop_backward_workspace_bytes(const mkg_hop_params* p, int64_t nnz) {
  return backward_layout(*p, nnz).total + 256;
}

int hop_backward(const mkg_graph* g, const mkg_frontier* fr, const float* w, const mkg_edge_factor* ef,
                 const mkg_hop_params* p, const mkg_coo3* g_ori, const mkg_coo3* g_inv, const mkg_coo3* g_ind,
                 const mkg_coo3* out_ori, const int64_t* arg_ori, const mkg_coo3* out_inv, const int64_t* arg_inv,
                 const int32_t* fhead, const int32_t* ftail, const int16_t* frel, float* grad_sp, float* grad_w,
                 float* grad_edge, void* ws, size_t ws_bytes, unsigned* err, cudaStream_t st) {
  int rc = check_hop_args(g, fr, w, ef, p);
  if (rc) return rc;
  MKG_REQUIRE(g_ori && g_inv && g_ind && grad_w && (grad_sp || fr->nnz == 0), "hop_backward: null argument");
  if (p->agg_mode == 1)
    MKG_REQUIRE(range_extent(*p) == p->E, "hop_backward: agg_mode 1 needs the full destination range");
  if (p->agg_mode == 1)
    MKG_REQUIRE(out_ori && out_inv && (arg_ori || out_ori->nnz == 0) && (arg_inv || out_inv->nnz == 0) &&
                    fhead && ftail && frel,
                "hop_backward: agg_mode 1 needs the forward outputs, their argmax facts and the fact table");
  HopLayout lay = backward_layout(*p, fr->nnz);
  if (lay.hash && (lay.capm > kMaxSlots || lay.capf > kMaxSlots)) {
    set_error("hop_backward: %lld messages per direction exceed one hash table (2^30 slots)",
              (long long)p->msg_bound);
    return MKG_ERR_CAPACITY;
  }
  MKG_REQUIRE(ws && ws_bytes >= lay.total, "hop_backward: workspace too small (%zu < %zu)", ws_bytes, lay.total);
  const bool merge = p->merge_outputs != 0;
  const mkg_coo3* gl[3] = {g_ori, g_inv, g_ind};
  if (lay.hash) {
    for (int k = 0; k < (merge ? 1 : 3); ++k)
      MKG_REQUIRE(gl[k]->nnz <= lay.slots(k) / 2, "hop_backward: %lld gradient keys exceed msg_bound",
                  (long long)gl[k]->nnz);
  }
  char* base = static_cast<char*>(ws);
  const int64_t F = fr->nnz;
  int32_t* lists = reinterpret_cast<int32_t*>(base + lay.off_lists);
  int32_t* counts = reinterpret_cast<int32_t*>(base + lay.off_counts);
  float* vals[3];
  KeyTable tabs[3];
  KeyTable map_tab = dense_table();
  int32_t* emap = p->agg_mode == 1 ? reinterpret_cast<int32_t*>(base + lay.off_map) : nullptr;
  if (!lay.hash) {
    float* gs = reinterpret_cast<float*>(base + lay.off_val);
    MKG_CUDA(cudaMemsetAsync(gs, 0, 4 * (size_t)lay.sval * 3, st));
    if (emap) MKG_CUDA(cudaMemsetAsync(emap, 0xff, 4 * (size_t)(p->B * p->L * p->E), st));
    for (int k = 0; k < 3; ++k) { vals[k] = gs + lay.sval * k; tabs[k] = dense_table(); }
  } else {
    unsigned long long* tkey = reinterpret_cast<unsigned long long*>(base + lay.off_tkey);
    float* tval = reinterpret_cast<float*>(base + lay.off_tval);
    const int64_t all = 2 * lay.capm + lay.capf;
    fill_u64_kernel<<<grid_for(all, 256, persistent_blocks(8)), 256, 0, st>>>(tkey, all, lay.empty());
    MKG_LAUNCHED("fill_u64_kernel");
    MKG_CUDA(cudaMemsetAsync(tval, 0, 4 * (size_t)all, st));
    for (int k = 0; k < 3; ++k) { vals[k] = tval + lay.base(k); tabs[k] = hash_table(tkey, lay, k); }
    if (emap) {
      unsigned long long* mkey = reinterpret_cast<unsigned long long*>(base + lay.off_mapkey);
      fill_u64_kernel<<<grid_for(lay.capf, 256, persistent_blocks(8)), 256, 0, st>>>(mkey, lay.capf, lay.empty());
      MKG_LAUNCHED("fill_u64_kernel");
      map_tab = KeyTable{mkey, lay.empty(), lay.capf - 1, 64 - log2_exact(lay.capf)};
    }
  }
  MKG_CUDA(cudaMemsetAsync(counts, 0, 16, st));
  const int64_t nw = p->B * p->L * p->n;
  double* gw64 = reinterpret_cast<double*>(base + lay.off_gw64);
  MKG_CUDA(cudaMemsetAsync(gw64, 0, 8 * (size_t)nw, st));
  double* gsp64 = reinterpret_cast<double*>(base + lay.off_gsp64);
  auto finish = [&]() -> int {  // grad_w and grad_sp = the fp64 sums rounded once
    round_gw_kernel<<<grid_for(nw, 256, persistent_blocks(2)), 256, 0, st>>>(gw64, nw, grad_w);
    MKG_LAUNCHED("round_gw_kernel");
    if (fr->nnz > 0) {
      round_gw_kernel<<<grid_for(fr->nnz, 256, persistent_blocks(2)), 256, 0, st>>>(gsp64, fr->nnz, grad_sp);
      MKG_LAUNCHED("round_gw_kernel");
    }
    return MKG_OK;
  };
  if (grad_edge) MKG_CUDA(cudaMemsetAsync(grad_edge, 0, 4 * (size_t)g->num_facts, st));
  if (merge) {  // one gradient store serves ori, inv and ind
    vals[1] = vals[2] = vals[0];
    tabs[1] = tabs[2] = tabs[0];
  }
  for (int k = 0; k < (merge ? 1 : 3); ++k) {
    if (gl[k]->nnz <= 0) continue;
    scatter_grad_kernel<<<grid_for(gl[k]->nnz, 256, persistent_blocks(8)), 256, 0, st>>>(
        *gl[k], p->B, p->L, range_lo(*p), range_extent(*p), tabs[k], vals[k], err);
    MKG_LAUNCHED("scatter_grad_kernel");
  }
  if (F == 0) return finish();
  HopCtx c = make_ctx(g, w, ef, p, err);
  Frontier f{fr->batch, fr->level, fr->entity, fr->value, F};
  backward_entry_init_kernel<<<grid_for(F, 256, persistent_blocks(8)), 256, 0, st>>>(
      f, c, tabs[2], vals[2], gsp64, gw64, map_tab, emap);
  MKG_LAUNCHED("backward_entry_init_kernel");
  if (p->agg_mode == 0) {
    classify_kernel<<<grid_for(F, 256, persistent_blocks(8)), 256, 0, st>>>(f, c, lists, counts, nullptr, nullptr,
                                                                             dense_table());
    MKG_LAUNCHED("classify_kernel");
    GradStore gs{{vals[0], vals[1]}, {tabs[0], tabs[1]}};
    bwd_tail_kernel<<<persistent_blocks(8), 256, 0, st>>>(f, c, lists, counts, gs, gsp64, gw64, grad_edge);
    bwd_mid_kernel<<<persistent_blocks(4), kMidWarps * 32, 0, st>>>(f, c, lists + F, counts + 1, gs, gsp64, gw64,
                                                                    grad_edge);
    bwd_hub_kernel<<<persistent_blocks(2), kHubThreads, 0, st>>>(f, c, lists + 2 * F, counts + 2, gs, gsp64, gw64,
                                                                 grad_edge);
    MKG_LAUNCHED("backward push kernels");
  } else {
    const mkg_coo3* outs[2] = {out_ori, out_inv};
    const int64_t* args[2] = {arg_ori, arg_inv};
    for (int d = 0; d < 2; ++d) {
      if (outs[d]->nnz <= 0) continue;
      bwd_argmax_kernel<<<grid_for(outs[d]->nnz, 256, persistent_blocks(8)), 256, 0, st>>>(
          d, *outs[d], args[d], f, c, tabs[d], vals[d], map_tab, emap, fhead, ftail, frel, gsp64, gw64,
          grad_edge);
      MKG_LAUNCHED("bwd_argmax_kernel");
    }
  }
  return finish();
}

}  // namespace mkg
