// The per-hop op behind FastLogFunctionSparse3DTopK: degree-bucketed push expansion of a
// sparse [B, L, E] frontier over the ori / inv CSR with the exact 256-bucket edge cap,
// reduced on the fly into key-major HBM slabs (sum: fp32 atomics + a hit byte per key;
// max: packed 64-bit (value, fact id) atomicMax), then compacted into coalesced COO in key
// order.  The backward walks the same messages and gathers the gradient from a dense slab.
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

size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

struct HopLayout {
  int64_t BLE, F, nblk;
  // per-slab strides in elements; every slab starts 256-byte aligned (the compaction
  // reads 16 hit bytes at a time as one uint4)
  int64_t sval, shit, spk;
  size_t off_val, off_hit, off_pk, off_lists, off_counts, off_blk, off_blkoff, off_cub, off_map, total;
  size_t cub_bytes;
};

size_t scan_bytes(int64_t nblk) {
  size_t b = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, b, (int64_t*)nullptr, (int64_t*)nullptr, (int)(nblk + 1));
  return b;
}

// Forward workspace: value slabs (sum: ori, inv, ind; max: ind), hit slabs, packed slabs
// (max: ori, inv), class lists, per-tile counts and offsets for the three outputs.
// Output entities: the destination range [lo, lo + extent) (the whole [0, E) by default).
int64_t range_lo(const mkg_hop_params& p) { return p.dst_hi > p.dst_lo ? p.dst_lo : 0; }
int64_t range_extent(const mkg_hop_params& p) { return p.dst_hi > p.dst_lo ? p.dst_hi - p.dst_lo : p.E; }

HopLayout forward_layout(const mkg_hop_params& p, int64_t F) {
  HopLayout L{};
  L.BLE = p.B * p.L * range_extent(p);
  L.F = F;
  L.nblk = (L.BLE + kTile - 1) / kTile;
  const int nval = p.agg_mode == 1 ? 1 : 3;
  L.sval = a256(4 * (size_t)L.BLE) / 4;
  L.shit = a256((size_t)L.BLE);
  L.spk = a256(8 * (size_t)L.BLE) / 8;
  size_t o = 0;
  L.off_val = o; o += 4 * (size_t)L.sval * nval;
  L.off_hit = o; o += (size_t)L.shit * nval;
  L.off_pk = o; o += p.agg_mode == 1 ? 8 * (size_t)L.spk * 2 : 0;
  L.off_lists = o; o += a256(4 * (size_t)(3 * F + 3));
  L.off_counts = o; o += a256(4 * 4);
  L.off_blk = o; o += a256(8 * (size_t)(L.nblk + 1) * 3);
  L.off_blkoff = o; o += a256(8 * (size_t)(L.nblk + 1) * 3);
  L.cub_bytes = scan_bytes(L.nblk);
  L.off_cub = o; o += a256(L.cub_bytes);
  L.off_map = 0;
  L.total = o;
  return L;
}

// Backward workspace: gradient slabs (ori, inv, ind), class lists, the key -> entry map.
HopLayout backward_layout(const mkg_hop_params& p, int64_t F) {
  HopLayout L{};
  L.BLE = p.B * p.L * range_extent(p);
  L.F = F;
  L.sval = a256(4 * (size_t)L.BLE) / 4;
  size_t o = 0;
  L.off_val = o; o += 4 * (size_t)L.sval * 3;
  L.off_lists = o; o += a256(4 * (size_t)(3 * F + 3));
  L.off_counts = o; o += a256(4 * 4);
  L.off_map = o; o += p.agg_mode == 1 ? a256(4 * (size_t)(p.B * p.L * p.E)) : 0;
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

// ------------------------------------------------------------------ message sinks
// Each sink receives one message: direction d, output key, value inputs and fact id.
struct SumSink {
  float* val[2];
  uint8_t* hit[2];
  __device__ __forceinline__ void msg(int d, int64_t key, float v, int64_t /*fact*/) {
    atomicAdd(val[d] + key, v);
    hit[d][key] = 1;
  }
};

struct MaxSink {
  unsigned long long* pk[2];
  __device__ __forceinline__ void msg(int d, int64_t key, float v, int64_t fact) {
    atomicMax(pk[d] + key, pack_value_rank(v, static_cast<uint32_t>(fact)));
  }
};

// Output key of (b, l, dst), or -1 when dst lies outside the destination range.
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
// emits its identity-channel message into the ind slab (sum).
__global__ void classify_kernel(Frontier f, HopCtx c, int32_t* __restrict__ lists,
                                int32_t* __restrict__ counts, float* __restrict__ ind_val,
                                uint8_t* __restrict__ ind_hit) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t base = warp0 * 32; base < f.F; base += nwarps * 32) {
    const int64_t i = base + lane;
    int cls = -1;
    if (i < f.F) {
      int64_t b, l, e;
      if (load_entry(f, c, i, b, l, e)) {
        const int64_t key = out_key0(c, b, l) + e;
        if (ind_val != nullptr && in_range(c, e)) {
          float v = c.wot_i ? 0.0f : f.v[i] * c.w[(b * c.L + l) * c.n + (c.n - 1)];
          atomicAdd(ind_val + key, v);
          ind_hit[key] = 1;
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

// ---------------------------------------------------------------- backward
// Incoming gradient keys must lie in the destination range (the forward produced no others).
__global__ void scatter_grad_kernel(mkg_coo3 g, int64_t B, int64_t L, int64_t lo, int64_t Eo,
                                    float* __restrict__ slab, unsigned* err) {
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < g.nnz;
       k += (int64_t)gridDim.x * blockDim.x) {
    int64_t b = g.indices[k], l = g.indices[g.nnz + k], e = g.indices[2 * g.nnz + k] - lo;
    if (b < 0 || b >= B || l < 0 || l >= L || e < 0 || e >= Eo) { raise_flag(err, MKG_DEV_BAD_KEY); continue; }
    atomicAdd(slab + (b * L + l) * Eo + e, g.values[k]);
  }
}

// Identity channel: grad_sp[i] = g_ind(key_i) * w[b,l,n-1] (initialises grad_sp) and
// grad_w[b,l,n-1] += g_ind * sv (fastlog.cu:2608-2644); also fills the key -> entry map.
__global__ void backward_entry_init_kernel(Frontier f, HopCtx c, const float* __restrict__ g_ind,
                                           float* __restrict__ grad_sp, float* __restrict__ grad_w,
                                           int32_t* __restrict__ entry_map) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < f.F;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t b, l, e;
    if (!load_entry(f, c, i, b, l, e)) { grad_sp[i] = 0.0f; continue; }
    if (entry_map) entry_map[(b * c.L + l) * c.E + e] = static_cast<int32_t>(i);
    float gsp = 0.0f;
    if (!c.wot_i && in_range(c, e)) {
      const int64_t wi = (b * c.L + l) * c.n + (c.n - 1);
      float g = g_ind[out_key0(c, b, l) + e];
      if (g != 0.0f) {
        gsp = g * c.w[wi];
        atomicAdd(grad_w + wi, g * f.v[i]);
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
  const float* gslab[2];
  float* grad_w;
  float* grad_edge;
  const EdgeFactor* f;
  float sv;
  int64_t key0, wbase;
  float acc;
  int64_t lo, Eo;
  __device__ __forceinline__ void operator()(int d, int64_t dst, int64_t ch, float wv, int64_t fact) {
    if (static_cast<uint64_t>(dst - lo) >= static_cast<uint64_t>(Eo)) return;  // another shard's destination
    float g = gslab[d][key0 + dst];
    if (g == 0.0f) return;
    float m = (*f)(fact);
    float gm = g * m;
    acc += gm * wv;
    atomicAdd(grad_w + wbase + ch, gm * sv);
    if (grad_edge) atomicAdd(grad_edge + fact, (((g * sv) * wv) * m) * edge_grad_factor(*f, fact));
  }
};

__global__ void bwd_tail_kernel(Frontier f, HopCtx c, const int32_t* __restrict__ list,
                                const int32_t* __restrict__ count, const float* gori, const float* ginv,
                                float* __restrict__ grad_sp, float* __restrict__ grad_w,
                                float* __restrict__ grad_edge) {
  const int64_t n = *count;
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n;
       k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = list[k];
    int64_t b, l, e;
    if (!load_entry(f, c, i, b, l, e)) continue;
    const float* wrow = c.w + (b * c.L + l) * c.n;
    BwdVisit vis{{gori, ginv}, grad_w, grad_edge, &c.factor, f.v[i], out_key0(c, b, l),
                 (b * c.L + l) * c.n, 0.0f, c.lo, c.Eo};
    for (int d = 0; d < 2; ++d) {
      const int64_t p0 = c.dir[d].row_ptr[e], p1 = c.dir[d].row_ptr[e + 1];
      for (int64_t p = p0; p < p1; ++p) visit_position(c, d, p, wrow, vis);
    }
    grad_sp[i] += vis.acc;
  }
}

__global__ void __launch_bounds__(kMidWarps * 32) bwd_mid_kernel(
    Frontier f, HopCtx c, const int32_t* __restrict__ list, const int32_t* __restrict__ count,
    const float* gori, const float* ginv, float* __restrict__ grad_sp, float* __restrict__ grad_w,
    float* __restrict__ grad_edge) {
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
    BwdVisit vis{{gori, ginv}, grad_w, grad_edge, &c.factor, f.v[i], out_key0(c, b, l),
                 (b * c.L + l) * c.n, 0.0f, c.lo, c.Eo};
    for (int d = 0; d < 2; ++d) {
      const int64_t p0 = c.dir[d].row_ptr[e], p1 = c.dir[d].row_ptr[e + 1];
      if (p1 - p0 <= c.cap) {
        for (int64_t p = p0 + lane; p < p1; p += 32) visit_position(c, d, p, wrow, vis);
      } else {
        warp_capped_direction(c, d, e, wrow, hist, vis);
      }
    }
    float tot = warp_sum(vis.acc);
    if (lane == 0) grad_sp[i] += tot;
  }
}

__global__ void __launch_bounds__(kHubThreads) bwd_hub_kernel(
    Frontier f, HopCtx c, const int32_t* __restrict__ list, const int32_t* __restrict__ count,
    const float* gori, const float* ginv, float* __restrict__ grad_sp, float* __restrict__ grad_w,
    float* __restrict__ grad_edge) {
  __shared__ float wstage[kHubStageMax];
  __shared__ int hist[kNumBuckets];
  __shared__ float part[kHubThreads / 32];
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
    BwdVisit vis{{gori, ginv}, grad_w, grad_edge, &c.factor, f.v[i], out_key0(c, b, l),
                 (b * c.L + l) * c.n, 0.0f, c.lo, c.Eo};
    for (int d = 0; d < 2; ++d) {
      const int64_t p0 = c.dir[d].row_ptr[e], p1 = c.dir[d].row_ptr[e + 1];
      if (p1 - p0 <= c.cap) {
        for (int64_t p = p0 + threadIdx.x; p < p1; p += blockDim.x) visit_position(c, d, p, wrow, vis);
      } else if (threadIdx.x < 32) {
        warp_capped_direction(c, d, e, wrow, hist, vis);
      }
    }
    float ws = warp_sum(vis.acc);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ws;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.0f;
      for (int q = 0; q < kHubThreads / 32; ++q) t += part[q];
      grad_sp[i] += t;
    }
    __syncthreads();
  }
}

// Max backward: the gradient of every output key goes to its argmax message only
// (fastlog_kernel.py:153-167 + fastlog.cu:2646-2676).
__global__ void bwd_argmax_kernel(int d, mkg_coo3 out, const int64_t* __restrict__ arg, Frontier f, HopCtx c,
                                  const float* __restrict__ gslab, const int32_t* __restrict__ entry_map,
                                  const int32_t* __restrict__ fhead, const int32_t* __restrict__ ftail,
                                  const int16_t* __restrict__ frel, float* __restrict__ grad_sp,
                                  float* __restrict__ grad_w, float* __restrict__ grad_edge) {
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < out.nnz;
       k += (int64_t)gridDim.x * blockDim.x) {
    int64_t b = out.indices[k], l = out.indices[out.nnz + k], dst = out.indices[2 * out.nnz + k];
    if (b < 0 || b >= c.B || l < 0 || l >= c.L || dst < 0 || dst >= c.E) { raise_flag(c.err, MKG_DEV_BAD_KEY); continue; }
    float g = gslab[(b * c.L + l) * c.E + dst];
    if (g == 0.0f) continue;
    int64_t fact = arg[k];
    if (fact < 0 || fact >= c.T) { raise_flag(c.err, MKG_DEV_BAD_FACT); continue; }
    int64_t src = d ? ftail[fact] : fhead[fact];
    int64_t ch = (d ? c.r_size : 0) + frel[fact];
    if (src < 0 || src >= c.E || ch < 0 || ch >= c.n - 1) { raise_flag(c.err, MKG_DEV_BAD_COL); continue; }
    int32_t i = entry_map[(b * c.L + l) * c.E + src];
    if (i < 0 || i >= f.F) { raise_flag(c.err, MKG_DEV_BAD_ENTRY); continue; }
    float m = c.factor(fact);
    float sv = f.v[i];
    int64_t wi = (b * c.L + l) * c.n + ch;
    float wv = c.w[wi];
    float gm = g * m;
    atomicAdd(grad_sp + i, gm * wv);
    atomicAdd(grad_w + wi, gm * sv);
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
  return MKG_OK;
}

}  // namespace

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
  MKG_REQUIRE(ws && ws_bytes >= lay.total, "hop_forward: workspace too small (%zu < %zu)", ws_bytes, lay.total);
  char* base = static_cast<char*>(ws);
  const int64_t BLE = lay.BLE, F = fr->nnz;
  float* val = reinterpret_cast<float*>(base + lay.off_val);
  uint8_t* hit = reinterpret_cast<uint8_t*>(base + lay.off_hit);
  unsigned long long* pk = reinterpret_cast<unsigned long long*>(base + lay.off_pk);
  int32_t* lists = reinterpret_cast<int32_t*>(base + lay.off_lists);
  int32_t* counts = reinterpret_cast<int32_t*>(base + lay.off_counts);
  int64_t* blk = reinterpret_cast<int64_t*>(base + lay.off_blk);
  int64_t* blkoff = reinterpret_cast<int64_t*>(base + lay.off_blkoff);
  void* cubtmp = base + lay.off_cub;
  const int nval = p->agg_mode == 1 ? 1 : 3;
  const int64_t SV = lay.sval, SH = lay.shit, SP = lay.spk;
  MKG_CUDA(cudaMemsetAsync(val, 0, 4 * (size_t)SV * nval, st));
  MKG_CUDA(cudaMemsetAsync(hit, 0, (size_t)SH * nval, st));
  if (p->agg_mode == 1) MKG_CUDA(cudaMemsetAsync(pk, 0, 8 * (size_t)SP * 2, st));
  MKG_CUDA(cudaMemsetAsync(counts, 0, 16, st));

  HopCtx c = make_ctx(g, w, ef, p, err);
  Frontier f{fr->batch, fr->level, fr->entity, fr->value, F};
  // ind slab: the last value slab (index 2 for sum, 0 for max)
  float* ind_val = val + SV * (nval - 1);
  uint8_t* ind_hit = hit + SH * (nval - 1);
  if (F > 0) {
    classify_kernel<<<grid_for(F, 256, persistent_blocks(8)), 256, 0, st>>>(f, c, lists, counts, ind_val, ind_hit);
    MKG_LAUNCHED("classify_kernel");
    const int tb = persistent_blocks(8), mb = persistent_blocks(4), hb = persistent_blocks(2);
    if (p->agg_mode == 0) {
      SumSink s{{val, val + SV}, {hit, hit + SH}};
      push_tail_kernel<SumSink><<<tb, 256, 0, st>>>(f, c, lists, counts, s);
      push_mid_kernel<SumSink><<<mb, kMidWarps * 32, 0, st>>>(f, c, lists + F, counts + 1, s);
      push_hub_kernel<SumSink><<<hb, kHubThreads, 0, st>>>(f, c, lists + 2 * F, counts + 2, s);
    } else {
      MaxSink s{{pk, pk + SP}};
      push_tail_kernel<MaxSink><<<tb, 256, 0, st>>>(f, c, lists, counts, s);
      push_mid_kernel<MaxSink><<<mb, kMidWarps * 32, 0, st>>>(f, c, lists + F, counts + 1, s);
      push_hub_kernel<MaxSink><<<hb, kHubThreads, 0, st>>>(f, c, lists + 2 * F, counts + 2, s);
    }
    MKG_LAUNCHED("push kernels");
  }
  // per-tile counts and offsets of the three outputs
  for (int which = 0; which < 3; ++which) {
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

int hop_emit(const mkg_hop_params* p, int64_t nnz, const void* ws, size_t ws_bytes, int which,
                   int64_t count, int64_t* indices, float* values, int64_t* arg, cudaStream_t st) {
  MKG_REQUIRE(p && ws, "hop_emit: null argument");
  MKG_REQUIRE(which >= 0 && which < 3, "hop_emit: which must be 0, 1 or 2");
  HopLayout lay = forward_layout(*p, nnz);
  MKG_REQUIRE(ws_bytes >= lay.total, "hop_emit: workspace too small");
  if (count == 0) return MKG_OK;
  MKG_REQUIRE(indices && values, "hop_emit: null output");
  const char* base = static_cast<const char*>(ws);
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
  MKG_REQUIRE(ws && ws_bytes >= lay.total, "hop_backward: workspace too small (%zu < %zu)", ws_bytes, lay.total);
  char* base = static_cast<char*>(ws);
  const int64_t BLE = lay.BLE, F = fr->nnz;
  float* gs = reinterpret_cast<float*>(base + lay.off_val);
  int32_t* lists = reinterpret_cast<int32_t*>(base + lay.off_lists);
  int32_t* counts = reinterpret_cast<int32_t*>(base + lay.off_counts);
  int32_t* emap = p->agg_mode == 1 ? reinterpret_cast<int32_t*>(base + lay.off_map) : nullptr;
  MKG_CUDA(cudaMemsetAsync(gs, 0, 4 * (size_t)lay.sval * 3, st));
  MKG_CUDA(cudaMemsetAsync(counts, 0, 16, st));
  if (emap) MKG_CUDA(cudaMemsetAsync(emap, 0xff, 4 * (size_t)BLE, st));
  MKG_CUDA(cudaMemsetAsync(grad_w, 0, 4 * (size_t)(p->B * p->L * p->n), st));
  if (grad_edge) MKG_CUDA(cudaMemsetAsync(grad_edge, 0, 4 * (size_t)g->num_facts, st));
  const mkg_coo3* gl[3] = {g_ori, g_inv, g_ind};
  for (int k = 0; k < 3; ++k) {
    if (gl[k]->nnz <= 0) continue;
    scatter_grad_kernel<<<grid_for(gl[k]->nnz, 256, persistent_blocks(8)), 256, 0, st>>>(
        *gl[k], p->B, p->L, range_lo(*p), range_extent(*p), gs + lay.sval * k, err);
    MKG_LAUNCHED("scatter_grad_kernel");
  }
  if (F == 0) return MKG_OK;
  HopCtx c = make_ctx(g, w, ef, p, err);
  Frontier f{fr->batch, fr->level, fr->entity, fr->value, F};
  backward_entry_init_kernel<<<grid_for(F, 256, persistent_blocks(8)), 256, 0, st>>>(
      f, c, gs + 2 * lay.sval, grad_sp, grad_w, emap);
  MKG_LAUNCHED("backward_entry_init_kernel");
  if (p->agg_mode == 0) {
    classify_kernel<<<grid_for(F, 256, persistent_blocks(8)), 256, 0, st>>>(f, c, lists, counts, nullptr, nullptr);
    MKG_LAUNCHED("classify_kernel");
    bwd_tail_kernel<<<persistent_blocks(8), 256, 0, st>>>(f, c, lists, counts, gs, gs + lay.sval, grad_sp, grad_w,
                                                          grad_edge);
    bwd_mid_kernel<<<persistent_blocks(4), kMidWarps * 32, 0, st>>>(f, c, lists + F, counts + 1, gs, gs + lay.sval,
                                                                    grad_sp, grad_w, grad_edge);
    bwd_hub_kernel<<<persistent_blocks(2), kHubThreads, 0, st>>>(f, c, lists + 2 * F, counts + 2, gs, gs + lay.sval,
                                                                 grad_sp, grad_w, grad_edge);
    MKG_LAUNCHED("backward push kernels");
  } else {
    const mkg_coo3* outs[2] = {out_ori, out_inv};
    const int64_t* args[2] = {arg_ori, arg_inv};
    for (int d = 0; d < 2; ++d) {
      if (outs[d]->nnz <= 0) continue;
      bwd_argmax_kernel<<<grid_for(outs[d]->nnz, 256, persistent_blocks(8)), 256, 0, st>>>(
          d, *outs[d], args[d], f, c, gs + lay.sval * d, emap, fhead, ftail, frel, grad_sp, grad_w, grad_edge);
      MKG_LAUNCHED("bwd_argmax_kernel");
    }
  }
  return MKG_OK;
}

}  // namespace mkg
