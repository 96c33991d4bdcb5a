// Key-slab hop engine: the uncapped sum hop of proof.py:569-609 on graphs whose frontiers are
// sparse but whose hops carry tens of millions of messages (the 4.6 M-entity and 86 M-entity
// shapes), where sorting or hashing the raw messages dominates.
//
// The output of a hop lives in a *slab store*: one fp32 slot per output key of a window of
// (b, l) rows x a destination range, plus one "touched" bit per slot.  A message adds its
// value to its slot with one atomicAdd; the thread whose add found the slot at zero sets the
// slot's bit.  The touched keys then come out in ascending key order by a popcount scan of the
// bitmap -- no sort, no hash table -- and the emit clears every slot and bit it read, so the
// store is all zeros again after each use (the caller zero-fills it once, when it is made).
//
// Messages of a frontier entry (b, l, s, x) are the records of push row s ({neighbour d,
// channel, fact, edge factor m}, grouped by channel), each worth (x * w[b, l, channel]) * m
// (fastlog.cu:2300-2318 order of operations), plus the identity message x * w[b, l, n - 1] to
// (b, l, s).  Work is cut into chunks of kChunkRecs records of one entry, dealt round-robin to
// the warps (measured on the 4.6 M-entity hop: 1.46 -> 1.11 ms against contiguous runs per warp).  Messages whose value is zero are not added: the hop loop drops
// zero values after its normalisation (drum.py:31-51), so they never reach its result.
//
// The backward walks the same chunks with the hop's output gradient held in the store as a
// lookup table: grad_sp[i] += g m w[ch], grad_w[b, l, ch] += (g m) x (fp64, one atomic per
// channel run of a warp), grad_edge[f] += g x w[ch] m dm/df (fastlog.cu:2551-2606,
// fastlog_kernel.py:1032-1098).
#include <cub/cub.cuh>

#include "mkg_common.cuh"

#define MKG_API extern "C" __attribute__((visibility("default")))

namespace mkg {
namespace {

constexpr int kChunkRecs = 128;           // push records per work chunk (4 per lane)
constexpr int kExpandThreads = 256;
constexpr int kTileThreads = 256;
constexpr int kWordsPerThread = 32;
constexpr int64_t kTileWords = (int64_t)kTileThreads * kWordsPerThread;  // bitmap words per collect block
constexpr int kRowBins = 256;             // row-sum bins of one emit / row-sum block

size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

struct Window {
  int64_t E, row0, nrows, lo, extent;
  __host__ __device__ int64_t slots() const { return nrows * extent; }
};

bool window_ok(const mkg_slab_window* w) {
  return w && w->E > 0 && w->row0 >= 0 && w->nrows > 0 && w->lo >= 0 && w->extent > 0 && w->lo + w->extent <= w->E;
}

Window make_window(const mkg_slab_window& w) { return Window{w.E, w.row0, w.nrows, w.lo, w.extent}; }

struct Store {
  float* val;
  uint32_t* bits;
};

Store make_store(void* base, int64_t slots) {
  Store s;
  s.val = static_cast<float*>(base);
  s.bits = reinterpret_cast<uint32_t*>(static_cast<char*>(base) + a256(4 * (size_t)slots));
  return s;
}

int64_t bitmap_words(int64_t slots) { return (slots + 31) / 32; }

// slot of a global key (row * E + e), with rows grouped by row_div (the sum over rules maps
// (b * L + l) to b with row_div = L); -1 when outside the window
__device__ __forceinline__ int64_t slot_of(const Window& w, int64_t key, int64_t row_div) {
  const int64_t row = (key / w.E) / row_div - w.row0;
  const int64_t e = key % w.E - w.lo;
  if (row < 0 || row >= w.nrows || e < 0 || e >= w.extent) return -1;
  return row * w.extent + e;
}

__device__ __forceinline__ void touch_add(const Store& s, int64_t slot, float v) {
  const float old = atomicAdd(s.val + slot, v);
  if (old == 0.0f) atomicOr(s.bits + (slot >> 5), 1u << (slot & 31));
}

// ------------------------------------------------------------------ chunking
__global__ void chunk_count_kernel(const int64_t* __restrict__ keys, int64_t nnz, int64_t E,
                                   const int32_t* __restrict__ push_ptr, int64_t* __restrict__ cnt, unsigned* err) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nnz; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = keys[i];
    int64_t c = 1;
    if (k < 0) {
      raise_flag(err, MKG_DEV_BAD_ENTRY);
    } else {
      const int64_t s = k % E;
      const int64_t deg = push_ptr[s + 1] - push_ptr[s];
      c = deg > kChunkRecs ? (deg + kChunkRecs - 1) / kChunkRecs : 1;  // >= 1: the identity message
    }
    cnt[i + 1] = c;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) cnt[0] = 0;
}

// entry owning chunk c: largest i with ptr[i] <= c
__device__ __forceinline__ int64_t chunk_entry(const int64_t* __restrict__ ptr, int64_t nnz, int64_t c) {
  int64_t lo = 0, hi = nnz - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (ptr[mid] <= c) lo = mid; else hi = mid - 1;
  }
  return lo;
}

struct ExpandArgs {
  const int32_t* push_ptr;
  const int4* push;          // mkg_adj_edge records
  const int64_t* keys;
  const float* vals;
  int64_t nnz;
  const int64_t* chunk_ptr;  // [nnz + 1]
  const float* w;            // [B * L, n]
  int64_t n;
  int identity;
  Window win;
  unsigned* err;
};

// ------------------------------------------------------------------ forward expansion
__global__ void __launch_bounds__(kExpandThreads) slab_expand_kernel(ExpandArgs a, Store st) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t total = a.chunk_ptr[a.nnz];
  // chunks round-robin over the warps: the chunks in flight at any time are consecutive, i.e.
  // a few (b, l) rows, whose touched slots stay in L2 while their atomics land
  for (int64_t c = warp; c < total; c += nwarps) {
    const int64_t i = chunk_entry(a.chunk_ptr, a.nnz, c);
    const int64_t key = a.keys[i];
    const int64_t row = key / a.win.E, s = key % a.win.E;
    const int64_t lrow = row - a.win.row0;
    if (lrow < 0 || lrow >= a.win.nrows) {  // entries must lie in the window's rows
      if (lane == 0) raise_flag(a.err, MKG_DEV_BAD_ENTRY);
      continue;
    }
    const float x = a.vals[i];
    const float* wrow = a.w + row * a.n;
    const int64_t k = c - a.chunk_ptr[i];
    if (k == 0 && lane == 0 && a.identity && s >= a.win.lo && s < a.win.lo + a.win.extent) {
      const float v = x * wrow[a.n - 1];
      if (v != 0.0f) touch_add(st, lrow * a.win.extent + (s - a.win.lo), v);
    }
    const int64_t rb = a.push_ptr[s] + k * kChunkRecs;
    const int64_t re = min(rb + kChunkRecs, (int64_t)a.push_ptr[s + 1]);
    if (x == 0.0f) continue;
    int4 rec[kChunkRecs / 32];
#pragma unroll
    for (int u = 0; u < kChunkRecs / 32; ++u) {
      const int64_t r = rb + u * 32 + lane;
      rec[u] = r < re ? a.push[r] : make_int4(-1, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kChunkRecs / 32; ++u) {
      const int d = rec[u].x, ch = rec[u].y;
      if (d < 0) continue;
      if (d >= a.win.E || ch < 0 || ch >= a.n - 1) { raise_flag(a.err, MKG_DEV_BAD_COL); continue; }
      const int64_t e = (int64_t)d - a.win.lo;
      if (e < 0 || e >= a.win.extent) continue;  // another rank's destination
      const float v = (x * __ldg(wrow + ch)) * __int_as_float(rec[u].w);
      if (v != 0.0f) touch_add(st, lrow * a.win.extent + e, v);
    }
  }
}

// ------------------------------------------------------------------ collect (count + emit)
__global__ void __launch_bounds__(kTileThreads) slab_count_kernel(const uint32_t* __restrict__ bits, int64_t words,
                                                                 int64_t* __restrict__ blk) {
  typedef cub::BlockReduce<int, kTileThreads> Reduce;
  __shared__ typename Reduce::TempStorage tmp;
  const int64_t w0 = blockIdx.x * kTileWords;
  int c = 0;
#pragma unroll 8
  for (int k = 0; k < kWordsPerThread; ++k) {
    const int64_t wi = w0 + (int64_t)k * kTileThreads + threadIdx.x;
    if (wi < words) c += __popc(bits[wi]);
  }
  const int total = Reduce(tmp).Sum(c);
  if (threadIdx.x == 0) blk[blockIdx.x] = total;
}

// Block b owns bitmap words [b * kTileWords, (b + 1) * kTileWords), visited 256 consecutive
// words at a time; a block scan of the popcounts places every set bit at its rank, so the
// keys come out in slot order = key order, and each word is cleared after it is read.  This
// pass only stores (no dependent loads per bit); slab_gather_kernel then reads the values.
__global__ void __launch_bounds__(kTileThreads) slab_emit_keys_kernel(Store st, Window win, int64_t words,
                                                                     const int64_t* __restrict__ blk_off,
                                                                     int64_t count, int64_t* __restrict__ keys_out) {
  typedef cub::BlockScan<int, kTileThreads> Scan;
  __shared__ typename Scan::TempStorage tmp;
  const int64_t w0 = blockIdx.x * kTileWords;
  int64_t base = blk_off[blockIdx.x];
  for (int k = 0; k < kWordsPerThread; ++k) {
    const int64_t wi = w0 + (int64_t)k * kTileThreads + threadIdx.x;
    uint32_t word = wi < words ? st.bits[wi] : 0u;
    int pos, tot;
    Scan(tmp).ExclusiveSum(__popc(word), pos, tot);
    __syncthreads();  // tmp reused next round
    if (word) {
      int64_t p = base + pos;
      st.bits[wi] = 0u;
      while (word) {
        const int j = __ffs(word) - 1;
        word &= word - 1;
        const int64_t slot = wi * 32 + j;
        const int64_t lrow = slot / win.extent;
        if (p < count) keys_out[p] = (win.row0 + lrow) * win.E + win.lo + (slot - lrow * win.extent);
        ++p;
      }
    }
    base += tot;
  }
}

// Values of the emitted keys: each thread takes kGatherItems consecutive outputs, issues their
// slot loads together, clears the slots and writes the values; row sums (optional, fp64) are
// collected per thread while the row stays the same, then in shared bins of the block's row
// span (global atomics when the span exceeds kRowBins rows).
constexpr int kGatherItems = 8;
__global__ void __launch_bounds__(kTileThreads) slab_gather_kernel(Store st, Window win,
                                                                  const int64_t* __restrict__ keys, int64_t count,
                                                                  float* __restrict__ vals_out,
                                                                  double* __restrict__ rsum) {
  __shared__ double bins[kRowBins];
  const int64_t i0 = blockIdx.x * (int64_t)kTileThreads * kGatherItems;
  if (i0 >= count) return;
  const int64_t i1 = min(i0 + (int64_t)kTileThreads * kGatherItems, count);
  const int64_t first_row = keys[i0] / win.E - win.row0;
  const int64_t span = keys[i1 - 1] / win.E - win.row0 - first_row + 1;
  const bool binned = rsum != nullptr && span <= kRowBins;
  if (binned)
    for (int i = threadIdx.x; i < kRowBins; i += kTileThreads) bins[i] = 0.0;
  __syncthreads();
  int64_t slot[kGatherItems], row[kGatherItems];
  float v[kGatherItems];
  const int64_t ib = i0 + (int64_t)threadIdx.x * kGatherItems;
#pragma unroll
  for (int u = 0; u < kGatherItems; ++u) {
    const int64_t i = ib + u;
    slot[u] = -1;
    row[u] = -1;
    if (i < i1) {
      const int64_t k = keys[i];
      row[u] = k / win.E - win.row0;
      slot[u] = row[u] * win.extent + (k % win.E - win.lo);
    }
  }
#pragma unroll
  for (int u = 0; u < kGatherItems; ++u) v[u] = slot[u] >= 0 ? st.val[slot[u]] : 0.0f;
  int64_t cur = -1;
  double acc = 0.0;
#pragma unroll
  for (int u = 0; u < kGatherItems; ++u) {
    if (slot[u] < 0) continue;
    st.val[slot[u]] = 0.0f;
    vals_out[ib + u] = v[u];
    if (rsum != nullptr) {
      if (row[u] != cur) {
        if (cur >= 0) {
          if (binned) atomicAdd(&bins[cur - first_row], acc);
          else atomicAdd(rsum + cur, acc);
        }
        cur = row[u];
        acc = 0.0;
      }
      acc += (double)v[u];
    }
  }
  if (rsum != nullptr && cur >= 0) {
    if (binned) atomicAdd(&bins[cur - first_row], acc);
    else atomicAdd(rsum + cur, acc);
  }
  if (binned) {
    __syncthreads();
    for (int i = threadIdx.x; i < span; i += kTileThreads)
      if (bins[i] != 0.0) atomicAdd(rsum + first_row + i, bins[i]);
  }
}

// ------------------------------------------------------------------ put / take
__global__ void slab_put_kernel(Store st, Window win, const int64_t* __restrict__ keys, const float* __restrict__ vals,
                                int64_t nnz, int64_t row_div, int mode, unsigned* err) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nnz; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = keys[i];
    const int64_t slot = k < 0 ? -1 : slot_of(win, k, row_div);
    if (slot < 0) { raise_flag(err, MKG_DEV_BAD_KEY); continue; }
    const float v = vals[i];
    if (mode == 0) st.val[slot] = v;
    else if (v != 0.0f) touch_add(st, slot, v);
  }
}

__global__ void slab_take_kernel(Store st, Window win, const int64_t* __restrict__ keys, int64_t nnz, int64_t row_div,
                                 float* __restrict__ out, int clear, unsigned* err) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nnz; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = keys[i];
    const int64_t slot = k < 0 ? -1 : slot_of(win, k, row_div);
    if (slot < 0) { raise_flag(err, MKG_DEV_BAD_KEY); if (out) out[i] = 0.0f; continue; }
    if (out) out[i] = st.val[slot];
    if (clear) st.val[slot] = 0.0f;
  }
}

// ------------------------------------------------------------------ backward expansion
__device__ __forceinline__ float grad_scale(const EdgeFactor& f, int64_t fact) {
  if (f.weight == nullptr) return 0.0f;
  const float ew = f.weight[fact];
  if (f.is_score) return 1.0f / fmaxf(ew, 1e-12f);
  const float z = -ew * f.scale;
  const float sg = static_cast<float>(1.0 / (1.0 + exp(static_cast<double>(z))));
  return f.scale * (1.0f - sg);
}

__global__ void __launch_bounds__(kExpandThreads) slab_expand_backward_kernel(
    ExpandArgs a, const float* __restrict__ gstore, EdgeFactor ef, int64_t num_facts, double* __restrict__ grad_sp,
    double* __restrict__ grad_w, float* __restrict__ grad_edge) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t total = a.chunk_ptr[a.nnz];
  // chunks round-robin over the warps: the chunks in flight at any time are consecutive, i.e.
  // a few (b, l) rows, whose touched slots stay in L2 while their atomics land
  for (int64_t c = warp; c < total; c += nwarps) {
    const int64_t i = chunk_entry(a.chunk_ptr, a.nnz, c);
    const int64_t key = a.keys[i];
    const int64_t row = key / a.win.E, s = key % a.win.E;
    const int64_t lrow = row - a.win.row0;
    if (lrow < 0 || lrow >= a.win.nrows) {
      if (lane == 0) raise_flag(a.err, MKG_DEV_BAD_ENTRY);
      continue;
    }
    const float x = a.vals[i];
    const float* wrow = a.w + row * a.n;
    double* gwrow = grad_w + row * a.n;
    const int64_t k = c - a.chunk_ptr[i];
    double gsp = 0.0;
    if (k == 0 && lane == 0 && a.identity && s >= a.win.lo && s < a.win.lo + a.win.extent) {
      const float g = gstore[lrow * a.win.extent + (s - a.win.lo)];
      if (g != 0.0f) {
        gsp += (double)(g * wrow[a.n - 1]);
        atomicAdd(gwrow + (a.n - 1), (double)(g * x));
      }
    }
    const int64_t rb = a.push_ptr[s] + k * kChunkRecs;
    const int64_t re = min(rb + kChunkRecs, (int64_t)a.push_ptr[s + 1]);
    int4 rec[kChunkRecs / 32];
#pragma unroll
    for (int u = 0; u < kChunkRecs / 32; ++u) {
      const int64_t r = rb + u * 32 + lane;
      rec[u] = r < re ? a.push[r] : make_int4(-1, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kChunkRecs / 32; ++u) {
      const int d = rec[u].x;
      int ch = rec[u].y;
      float g = 0.0f;
      bool live = d >= 0;
      if (live && (d >= a.win.E || ch < 0 || ch >= a.n - 1)) { raise_flag(a.err, MKG_DEV_BAD_COL); live = false; }
      const int64_t e = (int64_t)d - a.win.lo;
      if (live && (e < 0 || e >= a.win.extent)) live = false;
      if (live) g = gstore[lrow * a.win.extent + e];
      const float m = __int_as_float(rec[u].w);
      const float gm = g * m;
      float wv = 0.0f, part = 0.0f;
      if (live && gm != 0.0f) {
        wv = __ldg(wrow + ch);
        gsp += (double)(gm * wv);
        part = gm * x;
      }
      if (live && g != 0.0f && grad_edge != nullptr) {
        if (wv == 0.0f) wv = __ldg(wrow + ch);
        const int f = rec[u].z;
        if (f >= 0 && f < num_facts) {
          const float contrib = (((g * x) * wv) * m) * grad_scale(ef, f);
          if (contrib != 0.0f) atomicAdd(grad_edge + f, contrib);
        } else {
          raise_flag(a.err, MKG_DEV_BAD_FACT);
        }
      }
      // grad_w: records come grouped by channel, so a warp adds one fp64 partial per channel run
      if (!live) ch = -1;
      double dp = (double)part;
      const unsigned any = __ballot_sync(0xffffffffu, part != 0.0f);
      if (any) {
        const int prev = __shfl_up_sync(0xffffffffu, ch, 1);
        const bool head = lane == 0 || prev != ch;
        const unsigned heads = __ballot_sync(0xffffffffu, head);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const double y = __shfl_down_sync(0xffffffffu, dp, o);
          const int yc = __shfl_down_sync(0xffffffffu, ch, o);
          // add the partial of lane + o when it belongs to the same run (runs are contiguous)
          const unsigned between = (o + lane < 32) ? (heads >> (lane + 1)) & ((1u << o) - 1u) : 1u;
          if (lane + o < 32 && yc == ch && between == 0u) dp += y;
        }
        if (head && ch >= 0 && dp != 0.0) atomicAdd(gwrow + ch, dp);
      }
    }
    // entry gradient: one fp64 partial per warp and chunk
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) gsp += __shfl_xor_sync(0xffffffffu, gsp, o);
    if (lane == 0 && gsp != 0.0) atomicAdd(grad_sp + i, gsp);
  }
}

// ------------------------------------------------------------------ row sums
// out[row - row0] += sum of vals over the entries of that row; keys sorted ascending (rows
// contiguous), fp64 partials per thread run, shared bins per block span.
constexpr int kRowSumItems = 8;
__global__ void __launch_bounds__(kTileThreads) row_sums_kernel(const int64_t* __restrict__ keys, int64_t nnz, int64_t E,
                                                                int64_t row0, int64_t nrows,
                                                                const float* __restrict__ vals,
                                                                double* __restrict__ out, unsigned* err) {
  __shared__ double bins[kRowBins];
  const int64_t i0 = blockIdx.x * (int64_t)kTileThreads * kRowSumItems;
  const int64_t i1 = min(i0 + (int64_t)kTileThreads * kRowSumItems, nnz);
  if (i0 >= nnz) return;
  const int64_t first_row = keys[i0] / E - row0;
  const int64_t span = keys[i1 - 1] / E - row0 - first_row + 1;
  const bool binned = span >= 1 && span <= kRowBins;
  if (binned)
    for (int i = threadIdx.x; i < kRowBins; i += kTileThreads) bins[i] = 0.0;
  __syncthreads();
  int64_t cur = -1;
  double acc = 0.0;
  auto flush = [&]() {
    if (cur < 0) return;
    if (binned) atomicAdd(&bins[cur - first_row], acc);
    else atomicAdd(out + cur, acc);
  };
  // thread t takes items i0 + t * kRowSumItems ...: consecutive items share a row
  for (int u = 0; u < kRowSumItems; ++u) {
    const int64_t i = i0 + (int64_t)threadIdx.x * kRowSumItems + u;
    if (i >= i1) break;
    const int64_t r = keys[i] / E - row0;
    if (r < 0 || r >= nrows || (binned && (r < first_row || r >= first_row + span))) {
      raise_flag(err, MKG_DEV_BAD_KEY);
      continue;
    }
    if (r != cur) { flush(); cur = r; acc = 0.0; }
    acc += (double)vals[i];
  }
  flush();
  if (binned) {
    __syncthreads();
    for (int i = threadIdx.x; i < span; i += kTileThreads)
      if (bins[i] != 0.0) atomicAdd(out + first_row + i, bins[i]);
  }
}

__global__ void f64_to_f32_kernel(const double* __restrict__ in, int64_t n, float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = static_cast<float>(in[i]);
}

// ------------------------------------------------------------------ host helpers
size_t chunk_scan_bytes(int64_t nnz) {
  size_t b = 0;
  cub::DeviceScan::InclusiveSum(nullptr, b, (int64_t*)nullptr, (int64_t*)nullptr, (int)(nnz + 1));
  return b;
}

int64_t collect_blocks(int64_t slots) { return (bitmap_words(slots) + kTileWords - 1) / kTileWords; }

size_t collect_scan_bytes(int64_t nblk) {
  size_t b = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, b, (int64_t*)nullptr, (int64_t*)nullptr, (int)(nblk + 1));
  return b;
}

int build_chunks(const int32_t* push_ptr, const int64_t* keys, int64_t nnz, int64_t E, void* ws, size_t ws_bytes,
                 int64_t** chunk_ptr, unsigned* err, cudaStream_t st) {
  int64_t* cp = static_cast<int64_t*>(ws);
  void* temp = static_cast<char*>(ws) + a256(8 * (size_t)(nnz + 1));
  size_t tb = chunk_scan_bytes(nnz);
  MKG_REQUIRE(ws_bytes >= a256(8 * (size_t)(nnz + 1)) + tb, "slab: expand workspace too small");
  chunk_count_kernel<<<grid_for(nnz, 256, persistent_blocks(8)), 256, 0, st>>>(keys, nnz, E, push_ptr, cp, err);
  MKG_LAUNCHED("chunk_count_kernel");
  MKG_CUDA(cub::DeviceScan::InclusiveSum(temp, tb, cp, cp, (int)(nnz + 1), st));
  *chunk_ptr = cp;
  return MKG_OK;
}

int expand_grid(int64_t nnz) {
  (void)nnz;
  return persistent_blocks(8);
}

}  // namespace
}  // namespace mkg

using namespace mkg;

MKG_API size_t mkg_slab_store_bytes(int64_t slots) {
  if (slots <= 0) return 0;
  return a256(4 * (size_t)slots) + a256(4 * (size_t)bitmap_words(slots));
}

MKG_API size_t mkg_slab_expand_workspace_bytes(int64_t nnz) {
  if (nnz < 0) return 0;
  return a256(8 * (size_t)(nnz + 1)) + a256(chunk_scan_bytes(nnz));
}

MKG_API int mkg_slab_expand(const int32_t* push_ptr, const mkg_adj_edge* push, const int64_t* keys, const float* vals,
                            int64_t nnz, const float* w, int64_t n, int32_t identity, const mkg_slab_window* win,
                            void* store, void* workspace, size_t workspace_bytes, unsigned* dev_err,
                            mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(window_ok(win), "slab_expand: bad window");
  MKG_REQUIRE(nnz >= 0 && n >= 1 && n <= INT32_MAX, "slab_expand: bad sizes");
  if (nnz == 0) return MKG_OK;
  MKG_REQUIRE(push_ptr && push && keys && vals && w && store && workspace, "slab_expand: null argument");
  MKG_REQUIRE(nnz < INT32_MAX, "slab_expand: frontier of %lld entries exceeds the scan limit", (long long)nnz);
  int64_t* cp = nullptr;
  int rc = build_chunks(push_ptr, keys, nnz, win->E, workspace, workspace_bytes, &cp, dev_err, st);
  if (rc) return rc;
  ExpandArgs a{push_ptr, reinterpret_cast<const int4*>(push), keys, vals, nnz, cp, w, n, identity,
               make_window(*win), dev_err};
  slab_expand_kernel<<<expand_grid(nnz), kExpandThreads, 0, st>>>(a, make_store(store, win->nrows * win->extent));
  MKG_LAUNCHED("slab_expand_kernel");
  return MKG_OK;
}

MKG_API size_t mkg_slab_collect_workspace_bytes(int64_t slots) {
  if (slots <= 0) return 0;
  const int64_t nblk = collect_blocks(slots);
  return a256(8 * (size_t)(nblk + 1)) + a256(collect_scan_bytes(nblk));
}

MKG_API int mkg_slab_count(const mkg_slab_window* win, const void* store, void* workspace, size_t workspace_bytes,
                           int64_t* count_out, mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(window_ok(win) && store && workspace && count_out, "slab_count: bad argument");
  const int64_t slots = win->nrows * win->extent;
  const int64_t words = bitmap_words(slots), nblk = collect_blocks(slots);
  MKG_REQUIRE(nblk < INT32_MAX && workspace_bytes >= mkg_slab_collect_workspace_bytes(slots),
              "slab_count: workspace too small");
  int64_t* blk = static_cast<int64_t*>(workspace);
  void* temp = static_cast<char*>(workspace) + a256(8 * (size_t)(nblk + 1));
  size_t tb = collect_scan_bytes(nblk);
  Store s = make_store(const_cast<void*>(store), slots);
  MKG_CUDA(cudaMemsetAsync(blk + nblk, 0, sizeof(int64_t), st));
  slab_count_kernel<<<(unsigned)nblk, kTileThreads, 0, st>>>(s.bits, words, blk);
  MKG_LAUNCHED("slab_count_kernel");
  MKG_CUDA(cub::DeviceScan::ExclusiveSum(temp, tb, blk, blk, (int)(nblk + 1), st));
  MKG_CUDA(cudaMemcpyAsync(count_out, blk + nblk, sizeof(int64_t), cudaMemcpyDeviceToDevice, st));
  return MKG_OK;
}

MKG_API int mkg_slab_emit(const mkg_slab_window* win, void* store, const void* workspace, size_t workspace_bytes,
                          int64_t count, int64_t* keys_out, float* vals_out, double* row_sums, mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(window_ok(win) && store && workspace, "slab_emit: bad argument");
  MKG_REQUIRE(count >= 0 && (count == 0 || (keys_out && vals_out)), "slab_emit: bad output");
  const int64_t slots = win->nrows * win->extent;
  const int64_t words = bitmap_words(slots), nblk = collect_blocks(slots);
  MKG_REQUIRE(workspace_bytes >= mkg_slab_collect_workspace_bytes(slots), "slab_emit: workspace too small");
  const Store s = make_store(store, slots);
  slab_emit_keys_kernel<<<(unsigned)nblk, kTileThreads, 0, st>>>(s, make_window(*win), words,
                                                                 static_cast<const int64_t*>(workspace), count,
                                                                 keys_out);
  MKG_LAUNCHED("slab_emit_keys_kernel");
  if (count > 0) {
    const int64_t per = (int64_t)kTileThreads * kGatherItems;
    const int64_t gblocks = (count + per - 1) / per;
    MKG_REQUIRE(gblocks < INT32_MAX, "slab_emit: too many keys");
    slab_gather_kernel<<<(unsigned)gblocks, kTileThreads, 0, st>>>(s, make_window(*win), keys_out, count, vals_out,
                                                                     row_sums);
    MKG_LAUNCHED("slab_gather_kernel");
  }
  return MKG_OK;
}

MKG_API int mkg_slab_put(const mkg_slab_window* win, void* store, const int64_t* keys, const float* vals, int64_t nnz,
                         int64_t row_div, int32_t mode, unsigned* dev_err, mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(window_ok(win) && store && row_div >= 1 && (mode == 0 || mode == 1) && nnz >= 0, "slab_put: bad argument");
  if (nnz == 0) return MKG_OK;
  MKG_REQUIRE(keys && vals, "slab_put: null argument");
  slab_put_kernel<<<grid_for(nnz, 256, persistent_blocks(8)), 256, 0, st>>>(
      make_store(store, win->nrows * win->extent), make_window(*win), keys, vals, nnz, row_div, mode, dev_err);
  MKG_LAUNCHED("slab_put_kernel");
  return MKG_OK;
}

MKG_API int mkg_slab_take(const mkg_slab_window* win, void* store, const int64_t* keys, int64_t nnz, int64_t row_div,
                          float* out, int32_t clear, unsigned* dev_err, mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(window_ok(win) && store && row_div >= 1 && nnz >= 0, "slab_take: bad argument");
  if (nnz == 0) return MKG_OK;
  MKG_REQUIRE(keys, "slab_take: null argument");
  slab_take_kernel<<<grid_for(nnz, 256, persistent_blocks(8)), 256, 0, st>>>(
      make_store(store, win->nrows * win->extent), make_window(*win), keys, nnz, row_div, out, clear, dev_err);
  MKG_LAUNCHED("slab_take_kernel");
  return MKG_OK;
}

MKG_API int mkg_slab_expand_backward(const int32_t* push_ptr, const mkg_adj_edge* push, const int64_t* keys,
                                     const float* vals, int64_t nnz, const float* w, int64_t n, int32_t identity,
                                     const mkg_slab_window* win, const void* store, const mkg_edge_factor* ef,
                                     int64_t num_facts, double* grad_sp, double* grad_w, float* grad_edge,
                                     void* workspace, size_t workspace_bytes, unsigned* dev_err, mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(window_ok(win), "slab_expand_backward: bad window");
  MKG_REQUIRE(nnz >= 0 && n >= 1 && n <= INT32_MAX, "slab_expand_backward: bad sizes");
  if (nnz == 0) return MKG_OK;
  MKG_REQUIRE(push_ptr && push && keys && vals && w && store && ef && grad_sp && grad_w && workspace,
              "slab_expand_backward: null argument");
  MKG_REQUIRE(nnz < INT32_MAX, "slab_expand_backward: frontier too large");
  int64_t* cp = nullptr;
  int rc = build_chunks(push_ptr, keys, nnz, win->E, workspace, workspace_bytes, &cp, dev_err, st);
  if (rc) return rc;
  ExpandArgs a{push_ptr, reinterpret_cast<const int4*>(push), keys, vals, nnz, cp, w, n, identity,
               make_window(*win), dev_err};
  slab_expand_backward_kernel<<<expand_grid(nnz), kExpandThreads, 0, st>>>(
      a, static_cast<const float*>(store), make_factor(*ef), num_facts, grad_sp, grad_w, grad_edge);
  MKG_LAUNCHED("slab_expand_backward_kernel");
  return MKG_OK;
}

MKG_API int mkg_row_sums(const int64_t* keys, int64_t nnz, int64_t E, int64_t row0, int64_t nrows, const float* vals,
                         double* out, unsigned* dev_err, mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(E > 0 && nrows > 0 && row0 >= 0 && nnz >= 0, "row_sums: bad sizes");
  if (nnz == 0) return MKG_OK;
  MKG_REQUIRE(keys && vals && out, "row_sums: null argument");
  const int64_t per = (int64_t)kTileThreads * kRowSumItems;
  const int64_t blocks = (nnz + per - 1) / per;
  MKG_REQUIRE(blocks < INT32_MAX, "row_sums: too many entries");
  row_sums_kernel<<<(unsigned)blocks, kTileThreads, 0, st>>>(keys, nnz, E, row0, nrows, vals, out, dev_err);
  MKG_LAUNCHED("row_sums_kernel");
  return MKG_OK;
}

MKG_API int mkg_f64_to_f32(const double* in, int64_t n, float* out, mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(n >= 0 && (n == 0 || (in && out)), "f64_to_f32: bad argument");
  if (n == 0) return MKG_OK;
  f64_to_f32_kernel<<<grid_for(n, 256, persistent_blocks(8)), 256, 0, st>>>(in, n, out);
  MKG_LAUNCHED("f64_to_f32_kernel");
  return MKG_OK;
}
