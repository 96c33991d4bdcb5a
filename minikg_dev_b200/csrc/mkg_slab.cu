// Key-slab hop engine: the uncapped sum hop of proof.py:569-609 on graphs whose frontiers are
// sparse but whose hops carry tens of millions of messages (the 4.6 M-entity and 86 M-entity
// shapes), where sorting or hashing the raw messages dominates.
//
// The output of a hop lives in a *slab store*: one fp32 slot per output key of a window of
// (b, l) rows x a destination range, plus one "touched" bit per slot.  A message adds its
// value to its slot with one atomic reduction and sets the slot's bit with another (neither
// returns a value, so no thread waits on them).  The touched keys then come out in slot order
// (entity-major, below) by a popcount scan of the bitmap -- no sort, no hash table -- and the
// emit clears every slot and bit it read, so the
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
constexpr int kEmitStage = 128;           // keys a warp of the emit stages before writing them

size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

// Slots are entity-major: the window's rows of one destination are adjacent, so the rules of
// a query (rows b L .. b L + L - 1), which share their frontier entities and hence their
// destinations, land in one 32-byte sector of values and in one bitmap word.
struct Window {
  int64_t E, row0, nrows, lo, extent;
  FastDiv fe;  // key -> row
  __host__ __device__ int64_t slot(int64_t lrow, int64_t le) const { return le * nrows + lrow; }
};

bool window_ok(const mkg_slab_window* w) {
  return w && w->E > 0 && w->row0 >= 0 && w->nrows > 0 && w->lo >= 0 && w->extent > 0 && w->lo + w->extent <= w->E;
}

Window make_window(const mkg_slab_window& w) {
  return Window{w.E, w.row0, w.nrows, w.lo, w.extent, FastDiv::of(w.E)};
}

// row of a non-negative key divided by row_div (1, or L for the (b, e) keys of a sum over rules)
__device__ __forceinline__ int64_t div_rows(int64_t q, int64_t row_div) {
  if (row_div == 1) return q;
  return (q <= 0x7fffffff && row_div <= 0x7fffffff) ? (int64_t)((uint32_t)q / (uint32_t)row_div) : q / row_div;
}

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

// slot of a global key (row * E + e, key >= 0), with rows grouped by row_div (the sum over
// rules maps (b * L + l) to b with row_div = L); -1 when outside the window
__device__ __forceinline__ int64_t slot_of(const Window& w, int64_t key, int64_t row_div) {
  const int64_t q = w.fe.div(key);
  const int64_t row = div_rows(q, row_div) - w.row0;
  const int64_t e = key - q * w.E - w.lo;
  if (row < 0 || row >= w.nrows || e < 0 || e >= w.extent) return -1;
  return w.slot(row, e);
}


// Adds (sum) or raises to (max) a slot; returns the slot's previous value.  The max works on
// the float's bits as an unsigned integer, which orders non-negative floats correctly (the
// hop loop's messages are non-negative).
__device__ __forceinline__ float slot_accumulate(float* p, float v, int max_mode) {
  if (max_mode) return __uint_as_float(atomicMax(reinterpret_cast<unsigned*>(p), __float_as_uint(v)));
  return atomicAdd(p, v);
}

// The same without a returned value (a reduction the memory system completes on its own).
__device__ __forceinline__ void slot_reduce(float* p, float v, int max_mode) {
  if (max_mode) atomicMax(reinterpret_cast<unsigned*>(p), __float_as_uint(v));
  else atomicAdd(p, v);
}

__device__ __forceinline__ void touch_add(const Store& s, int64_t slot, float v, int max_mode = 0) {
  const float old = slot_accumulate(s.val + slot, v, max_mode);
  if (old == 0.0f) atomicOr(s.bits + (slot >> 5), 1u << (slot & 31));
}

// ------------------------------------------------------------------ chunking
// The push lists of a launch: one per destination tile (records of the tile's destinations
// only).  A launch walks work items (tile t, frontier entry i), tile-major, so the chunks in
// flight at any time belong to one tile and touch only its part of the store.
constexpr int kMaxTiles = MKG_SLAB_MAX_TILES;
struct TileLists {
  const int32_t* ptr[kMaxTiles];
  const int4* push[kMaxTiles];  // mkg_adj_edge records
  int count;
};

// tile t's lists, selected with constant indices (the parameter arrays stay in constant space)
__device__ __forceinline__ void tile_lists(const TileLists& tl, int t, const int32_t*& ptr, const int4*& push) {
  ptr = tl.ptr[0];
  push = tl.push[0];
#pragma unroll
  for (int q = 1; q < kMaxTiles; ++q)
    if (t == q) { ptr = tl.ptr[q]; push = tl.push[q]; }
}

// work item j = t * nnz + i -> (t, i); t < kMaxTiles
__device__ __forceinline__ int split_item(int64_t j, int64_t nnz, int64_t& i) {
  int t = 0;
  while (j >= nnz && t < kMaxTiles - 1) { j -= nnz; ++t; }
  i = j;
  return t;
}

// Chunks per work item (tile t, entry i): its records in tile t in chunks of kChunkRecs, and
// one chunk for the identity message alone (tile 0, when the launch adds identity messages)
// where it has none.  An entry of a row outside the window's rows gets none (the frontier of
// a windowed hop is passed whole to every window), a negative key none and a flag.
__global__ void chunk_count_kernel(const int64_t* __restrict__ keys, int64_t nnz, int64_t E, int64_t row0,
                                   int64_t nrows, TileLists tl, int identity, int64_t* __restrict__ cnt,
                                   unsigned long long* __restrict__ next, unsigned* err) {
  const int64_t items = nnz * tl.count;
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < items; j += (int64_t)gridDim.x * blockDim.x) {
    int64_t i;
    const int t = split_item(j, nnz, i);
    const int64_t k = keys[i];
    int64_t c = 0;
    if (k < 0) {
      if (t == 0) raise_flag(err, MKG_DEV_BAD_ENTRY);
    } else if (k / E - row0 >= 0 && k / E - row0 < nrows) {
      const int64_t s = k % E;
      const int32_t* pp;
      const int4* pr;
      tile_lists(tl, t, pp, pr);
      const int64_t deg = pp[s + 1] - pp[s];
      c = deg > 0 ? (deg + kChunkRecs - 1) / kChunkRecs : (t == 0 && identity ? 1 : 0);
    }
    cnt[j + 1] = c;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    cnt[0] = 0;
    *next = 0ull;  // the walk's work counter
  }
}

// Chunks are handed out in order from one counter, kGrab consecutive ones per warp at a time, so
// the chunks in flight at any time are consecutive (one tile, a few (b, l) rows) however the
// blocks are scheduled.  Measured on the 4.6 M-entity step against the static round-robin:
// one chunk per grab serialised on the counter's address (forward / backward 2.46 / 2.11 ms per
// hop against 1.94 / 1.66); four per grab gave 1.74 / 1.42 ms.
constexpr int kGrab = 4;
__device__ __forceinline__ int64_t grab_chunks(unsigned long long* next, int lane) {
  unsigned long long c = 0;
  if (lane == 0) c = atomicAdd(next, (unsigned long long)kGrab);
  return static_cast<int64_t>(__shfl_sync(0xffffffffu, c, 0));
}

// the warp's next chunk: the next of its batch [base, base + kGrab), or the first of a new one
__device__ __forceinline__ int64_t next_chunk(unsigned long long* next, int lane, int64_t& base, int& k) {
  if (++k == kGrab) {
    k = 0;
    base = grab_chunks(next, lane);
  }
  return base + k;
}

// entry owning chunk c: largest i with ptr[i] <= c
__device__ __forceinline__ int64_t chunk_entry(const int64_t* __restrict__ ptr, int64_t nnz, int64_t c) {
  int64_t lo = 0, hi = nnz - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (__ldg(ptr + mid) <= c) lo = mid; else hi = mid - 1;  // read-only path: the top levels stay in L1
  }
  return lo;
}

struct ExpandArgs {
  TileLists tiles;
  const int64_t* keys;
  const float* vals;
  int64_t nnz;               // frontier entries
  const int64_t* chunk_ptr;  // [tiles.count * nnz + 1]
  unsigned long long* next;  // work counter (zeroed by the chunk count)
  const float* w;            // [B * L, n]
  int64_t n;
  int identity;
  int max_mode;              // 1: slots keep the largest message (values must be >= 0)
  Window win;
  unsigned* err;
  double* rsum;              // forward, sum mode, may be null: [nrows] row sums of the added messages
};

// ------------------------------------------------------------------ forward expansion
__global__ void __launch_bounds__(kExpandThreads, 5) slab_expand_kernel(ExpandArgs a, Store st) {
  const int lane = threadIdx.x & 31;
  const int64_t items = a.nnz * a.tiles.count;
  const int64_t total = a.chunk_ptr[items];
  // chunks in order from the work counter: the chunks in flight at any time are consecutive,
  // i.e. one tile and a few (b, l) rows, whose touched slots stay in L2 while their atomics land
  int64_t cbase = grab_chunks(a.next, lane);
  int ck = 0;
  for (int64_t c = cbase; c < total; c = next_chunk(a.next, lane, cbase, ck)) {
    const int64_t j = chunk_entry(a.chunk_ptr, items, c);
    int64_t i;
    const int t = split_item(j, a.nnz, i);
    const int64_t key = a.keys[i];
    const int64_t row = key / a.win.E, s = key % a.win.E;
    const int64_t lrow = row - a.win.row0;
    if (lrow < 0 || lrow >= a.win.nrows) {  // entries must lie in the window's rows
      if (lane == 0) raise_flag(a.err, MKG_DEV_BAD_ENTRY);
      continue;
    }
    const int32_t* push_ptr;
    const int4* push;
    tile_lists(a.tiles, t, push_ptr, push);
    const float x = a.vals[i];
    const float* wrow = a.w + row * a.n;
    const int64_t k = c - a.chunk_ptr[j];
    double part = 0.0;  // the lane's added message values (the row sum of the normalisation)
    if (k == 0 && t == 0 && lane == 0 && a.identity && s >= a.win.lo && s < a.win.lo + a.win.extent) {
      const float v = x * wrow[a.n - 1];
      if (v != 0.0f) {
        const int64_t sl = a.win.slot(lrow, s - a.win.lo);
        slot_reduce(st.val + sl, v, a.max_mode);
        atomicOr(st.bits + (sl >> 5), 1u << (sl & 31));
        part += (double)v;
      }
    }
    const int64_t rb = push_ptr[s] + k * kChunkRecs;
    const int64_t re = min(rb + kChunkRecs, (int64_t)push_ptr[s + 1]);
    if (x != 0.0f) {
    int4 rec[kChunkRecs / 32];
#pragma unroll
    for (int u = 0; u < kChunkRecs / 32; ++u) {
      const int64_t r = rb + u * 32 + lane;
      rec[u] = r < re ? push[r] : make_int4(-1, 0, 0, 0);
    }
    // the lane's records in two rounds: all rule-weight loads in flight, then the reductions
    constexpr int kU = kChunkRecs / 32;
    int64_t slot[kU];
    float wv[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int d = rec[u].x, ch = rec[u].y;
      slot[u] = -1;
      wv[u] = 0.0f;
      if (d < 0) continue;
      if (d >= a.win.E || ch < 0 || ch >= a.n - 1) { raise_flag(a.err, MKG_DEV_BAD_COL); continue; }
      const int64_t e = (int64_t)d - a.win.lo;
      if (e < 0 || e >= a.win.extent) continue;  // another rank's destination
      slot[u] = a.win.slot(lrow, e);
      wv[u] = __ldg(wrow + ch);
    }
    // fire-and-forget reductions: no add waits for the slot's old value; every add also sets
    // its slot's bit (setting it again is harmless)
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const float v = (x * wv[u]) * __int_as_float(rec[u].w);
      if (slot[u] >= 0 && v != 0.0f) {
        slot_reduce(st.val + slot[u], v, a.max_mode);
        atomicOr(st.bits + (slot[u] >> 5), 1u << (slot[u] & 31));
        part += (double)v;
      }
    }
    }
    // one fp64 row-sum atomic per chunk: every message of a chunk lies in its entry's row
    if (a.rsum != nullptr) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (lane == 0 && part != 0.0) atomicAdd(a.rsum + lrow, part);
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

// Block b owns bitmap words [b * kTileWords, (b + 1) * kTileWords) (the tile slab_count_kernel
// counted); every set bit is placed at its rank, so the keys come out in slot order
// (entity-major), and each word is cleared after it is read.
__global__ void __launch_bounds__(kTileThreads) slab_emit_kernel(Store st, Window win, int64_t words,
                                                                const int64_t* __restrict__ blk_off, int64_t count,
                                                                int64_t* __restrict__ keys_out) {
  // warp w of the block owns the tile's words [w * 1024, (w + 1) * 1024), lane l reads words
  // w * 1024 + k * 32 + l: one pass counts the warp's bits, a scan of the 8 warp counts in
  // shared memory places each warp, a second pass emits with a warp scan per 32 words
  constexpr int kWarps = kTileThreads / 32;
  constexpr int kSpan = (int)(kTileWords / kWarps);  // words per warp
  __shared__ long long warp_base[kWarps];
  __shared__ uint32_t wsm[kWarps][kSpan];  // the warp's words, loaded once (all loads in flight)
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t wb = blockIdx.x * kTileWords + (int64_t)wid * kSpan;
  int c = 0;
#pragma unroll 8
  for (int k = 0; k < kSpan / 32; ++k) {
    const int64_t wi = wb + k * 32 + lane;
    const uint32_t wv = wi < words ? st.bits[wi] : 0u;
    wsm[wid][k * 32 + lane] = wv;
    c += __popc(wv);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if (lane == 0) warp_base[wid] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    long long run = blk_off[blockIdx.x];
    for (int w = 0; w < kWarps; ++w) {
      const long long t = warp_base[w];
      warp_base[w] = run;
      run += t;
    }
  }
  __syncthreads();
  // The slots of 32 words (up to 1024 set bits) are placed in a per-warp shared buffer at their
  // rank, kEmitStage at a time; the whole warp then writes their keys (coalesced stores even
  // where the entity-major bitmap packs many bits into neighbouring words).  The values are
  // left to slab_gather_kernel: loading them here put one memory round trip behind every
  // non-empty group of words (measured: 1.0 -> 3.2 ms per launch on the 4.6 M-entity hop).
  __shared__ long long stage[kWarps][kEmitStage];
  const FastDiv win_rows = FastDiv::of(win.nrows);  // slot -> entity
  int64_t base = warp_base[wid];
  for (int k = 0; k < kSpan / 32; ++k) {
    const uint32_t word0 = wsm[wid][k * 32 + lane];
    if (__ballot_sync(0xffffffffu, word0 != 0u) == 0u) continue;  // most groups are empty
    const int64_t wi = wb + k * 32 + lane;
    const int pc = __popc(word0);
    int incl = pc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int tot = __shfl_sync(0xffffffffu, incl, 31);
    if (word0) st.bits[wi] = 0u;
    for (int pass = 0; pass < tot; pass += kEmitStage) {
      uint32_t word = word0;
      int q = incl - pc;  // rank of the lane's first bit among the 32 words' bits
      while (word) {
        const int j = __ffs(word) - 1;
        word &= word - 1;
        if (q >= pass && q < pass + kEmitStage) stage[wid][q - pass] = wi * 32 + j;
        ++q;
      }
      __syncwarp();
      const int m = tot - pass < kEmitStage ? tot - pass : kEmitStage;
      for (int t = lane; t < m; t += 32) {
        const int64_t p = base + pass + t;
        const int64_t sl = stage[wid][t];
        const int64_t le = win_rows.div(sl);
        if (p < count) keys_out[p] = (win.row0 + (sl - le * win.nrows)) * win.E + win.lo + le;
      }
      __syncwarp();
    }
    base += tot;
  }
}

// Values of the emitted keys: a block walks tiles of kTileThreads * kGatherItems outputs, each
// thread kGatherItems of them a block width apart (neighbouring lanes read neighbouring keys
// and, in the entity-major store, neighbouring slots), issues their slot loads together, clears
// the slots and writes the values.
constexpr int kGatherItems = 8;

// The sum hop's mass normalisation applied as the values are gathered (NORM): x = (y / d) *
// min(d, 1) with d the key's row sum (fp32 division and product, as mass_norm_kernel), and the
// count of results the loop then drops (zero, or under a positive threshold).
struct GatherNorm {
  const float* d;  // [nrows] row sums of the window's rows
  float thr;
  float* x;        // [count]
  unsigned long long* dropped;
};

template <bool NORM>
__global__ void __launch_bounds__(kTileThreads) slab_gather_kernel(Store st, Window win,
                                                                  const int64_t* __restrict__ keys, int64_t count,
                                                                  float* __restrict__ vals_out, GatherNorm nm) {
  constexpr int64_t kTile = (int64_t)kTileThreads * kGatherItems;
  unsigned long long drop = 0;
  for (int64_t i0 = blockIdx.x * kTile; i0 < count; i0 += (int64_t)gridDim.x * kTile) {
    int64_t slot[kGatherItems];
    float dr[kGatherItems];  // NORM: the key's row sum, loaded with the slot (its latency overlaps)
    float v[kGatherItems];
#pragma unroll
    for (int u = 0; u < kGatherItems; ++u) {
      const int64_t i = i0 + u * kTileThreads + threadIdx.x;
      slot[u] = -1;
      dr[u] = 1.0f;
      if (i < count) {
        const int64_t k = keys[i];
        const int64_t q = win.fe.div(k);
        if (NORM) dr[u] = nm.d[q - win.row0];
        slot[u] = win.slot(q - win.row0, k - q * win.E - win.lo);
      }
    }
#pragma unroll
    for (int u = 0; u < kGatherItems; ++u) v[u] = slot[u] >= 0 ? st.val[slot[u]] : 0.0f;
#pragma unroll
    for (int u = 0; u < kGatherItems; ++u) {
      if (slot[u] < 0) continue;
      st.val[slot[u]] = 0.0f;
      vals_out[i0 + u * kTileThreads + threadIdx.x] = v[u];
    }
    if (NORM) {  // after the stores: the slots no longer live while the divisions run
#pragma unroll
      for (int u = 0; u < kGatherItems; ++u) {
        const int64_t i = i0 + u * kTileThreads + threadIdx.x;
        if (i >= count) continue;
        const float x = __fdiv_rn(v[u], dr[u]) * fminf(dr[u], 1.0f);
        nm.x[i] = x;
        if (x == 0.0f || (nm.thr > 0.0f && x < nm.thr)) ++drop;
      }
    }
  }
  if (NORM) {
    drop = __reduce_add_sync(0xffffffffu, static_cast<unsigned>(drop));
    if ((threadIdx.x & 31) == 0 && drop) atomicAdd(nm.dropped, drop);
  }
}

constexpr int kMaxBinRows = 2048;  // 16 KB of fp64 row bins per block (gradient row sums)

// ------------------------------------------------------------------ put / take
__global__ void slab_put_kernel(Store st, Window win, const int64_t* __restrict__ keys, const float* __restrict__ vals,
                                int64_t nnz, int64_t row_div, int mode, unsigned* err) {
  const bool skip_outside = (mode & MKG_SLAB_SKIP_OUTSIDE) != 0;
  const int op = mode & 3;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nnz; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = keys[i];
    const int64_t slot = k < 0 ? -1 : slot_of(win, k, row_div);
    if (slot < 0) {
      if (!(skip_outside && k >= 0)) raise_flag(err, MKG_DEV_BAD_KEY);
      continue;
    }
    const float v = vals[i];
    if (op == 0) st.val[slot] = v;
    else if (v != 0.0f) touch_add(st, slot, v, op == 2);
  }
}

// out (may be NULL) receives the slot values of the keys; keys skipped as another window's
// (MKG_SLAB_SKIP_OUTSIDE) leave their out entry as it was
__global__ void slab_take_kernel(Store st, Window win, const int64_t* __restrict__ keys, int64_t nnz, int64_t row_div,
                                 float* __restrict__ out, int clear, unsigned* err) {
  const bool skip_outside = (clear & MKG_SLAB_SKIP_OUTSIDE) != 0;
  const bool zero = (clear & 1) != 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nnz; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = keys[i];
    const int64_t slot = k < 0 ? -1 : slot_of(win, k, row_div);
    if (slot < 0) {
      if (skip_outside && k >= 0) continue;
      raise_flag(err, MKG_DEV_BAD_KEY);
      if (out) out[i] = 0.0f;
      continue;
    }
    if (out) out[i] = st.val[slot];
    if (zero) st.val[slot] = 0.0f;
  }
}

// ------------------------------------------------------------------ backward expansion
// d m / d weight divided out of m, from the record's own factor m = [mask] * score: where the
// mask is on, m is the score itself (weight, or sigmoid(weight * scale) rounded to fp32), so
// 1 / max(weight, 1e-12) = 1 / max(m, 1e-12) and scale * (1 - sigmoid) = scale * (1 - m); where
// it is off m = 0 and the contribution is zero either way.  No per-message read of the weights.
__device__ __forceinline__ float grad_scale(const EdgeFactor& f, float m) {
  if (f.weight == nullptr) return 0.0f;
  if (f.is_score) return 1.0f / fmaxf(m, 1e-12f);
  return f.scale * (1.0f - m);
}

__global__ void __launch_bounds__(kExpandThreads) slab_expand_backward_kernel(
    ExpandArgs a, const float* __restrict__ gstore, EdgeFactor ef, int64_t num_facts, double* __restrict__ grad_sp,
    double* __restrict__ grad_w, float* __restrict__ grad_edge) {
  const int lane = threadIdx.x & 31;
  const int64_t items = a.nnz * a.tiles.count;
  const int64_t total = a.chunk_ptr[items];
  // chunks in order from the work counter: the chunks in flight at any time are consecutive,
  // i.e. one tile and a few (b, l) rows, whose touched slots stay in L2 while their loads land
  int64_t cbase = grab_chunks(a.next, lane);
  int ck = 0;
  for (int64_t c = cbase; c < total; c = next_chunk(a.next, lane, cbase, ck)) {
    const int64_t j = chunk_entry(a.chunk_ptr, items, c);
    int64_t i;
    const int t = split_item(j, a.nnz, i);
    const int64_t key = a.keys[i];
    const int64_t row = key / a.win.E, s = key % a.win.E;
    const int64_t lrow = row - a.win.row0;
    if (lrow < 0 || lrow >= a.win.nrows) {
      if (lane == 0) raise_flag(a.err, MKG_DEV_BAD_ENTRY);
      continue;
    }
    const int32_t* push_ptr;
    const int4* push;
    tile_lists(a.tiles, t, push_ptr, push);
    const float x = a.vals[i];
    const float* wrow = a.w + row * a.n;
    double* gwrow = grad_w + row * a.n;
    const int64_t k = c - a.chunk_ptr[j];
    double gsp = 0.0;
    if (k == 0 && t == 0 && lane == 0 && a.identity && s >= a.win.lo && s < a.win.lo + a.win.extent) {
      const float g = gstore[a.win.slot(lrow, s - a.win.lo)];
      if (g != 0.0f) {
        gsp += (double)g * (double)wrow[a.n - 1];
        atomicAdd(gwrow + (a.n - 1), (double)g * (double)x);
      }
    }
    const int64_t rb = push_ptr[s] + k * kChunkRecs;
    const int64_t re = min(rb + kChunkRecs, (int64_t)push_ptr[s + 1]);
    int4 rec[kChunkRecs / 32];
#pragma unroll
    for (int u = 0; u < kChunkRecs / 32; ++u) {
      const int64_t r = rb + u * 32 + lane;
      rec[u] = r < re ? push[r] : make_int4(-1, 0, 0, 0);
    }
    // all of the lane's gradient lookups and rule-weight loads go out before any is used
    constexpr int kU = kChunkRecs / 32;
    float gl[kU], wl[kU];
    bool lv[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int d = rec[u].x, ch = rec[u].y;
      bool live = d >= 0;
      if (live && (d >= a.win.E || ch < 0 || ch >= a.n - 1)) { raise_flag(a.err, MKG_DEV_BAD_COL); live = false; }
      const int64_t e = (int64_t)d - a.win.lo;
      if (live && (e < 0 || e >= a.win.extent)) live = false;
      lv[u] = live;
      gl[u] = live ? gstore[a.win.slot(lrow, e)] : 0.0f;
      wl[u] = live ? __ldg(wrow + ch) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      int ch = rec[u].y;
      const bool live = lv[u];
      const float g = gl[u];
      const float m = __int_as_float(rec[u].w);
      const float wv = wl[u];
      // the products in fp64 (each exact): the rule-weight and entry gradients are sums whose
      // terms cancel, where fp32-rounded terms drifted past 1e-5 of the result
      const double gm = (double)g * (double)m;
      double dp = 0.0;
      if (live && gm != 0.0) {
        gsp += gm * (double)wv;
        dp = gm * (double)x;
      }
      if (live && g != 0.0f && grad_edge != nullptr) {
        const int f = rec[u].z;
        if (f >= 0 && f < num_facts) {
          const float contrib = (((g * x) * wv) * m) * grad_scale(ef, m);
          if (contrib != 0.0f) atomicAdd(grad_edge + f, contrib);
        } else {
          raise_flag(a.err, MKG_DEV_BAD_FACT);
        }
      }
      // grad_w: records come grouped by channel, so a warp adds one fp64 partial per channel run
      if (!live) ch = -1;
      const unsigned any = __ballot_sync(0xffffffffu, dp != 0.0);
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

// ------------------------------------------------------------------ mass normalisation
// normalize_sparse3d(.., 0, "mass") on a key-sorted state (drum.py:31-51): x = (y / d) *
// min(d, 1) with d the row's sum (fp32 division and product, as torch computes them); counts
// the zeros the result holds (entries the hop loop then drops) and the entries under a state
// threshold.
__global__ void mass_norm_kernel(const int64_t* __restrict__ keys, const float* __restrict__ y, int64_t n, FastDiv E,
                                 int64_t row0, int64_t nrows, const float* __restrict__ d, float thr,
                                 float* __restrict__ x, unsigned long long* __restrict__ dropped, unsigned* err) {
  unsigned long long local = 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = E.div(keys[i]) - row0;
    float v = 0.0f;
    if (r < 0 || r >= nrows) {
      raise_flag(err, MKG_DEV_BAD_KEY);
    } else {
      const float dr = d[r];
      v = __fdiv_rn(y[i], dr) * fminf(dr, 1.0f);
    }
    x[i] = v;
    if (v == 0.0f || (thr > 0.0f && v < thr)) ++local;
  }
  local = __reduce_add_sync(0xffffffffu, (unsigned)local);
  if ((threadIdx.x & 31) == 0 && local) atomicAdd(dropped, local);
}

// Row sums of the normalisation gradient's two terms (fp64): sums[0][r] += gx * q and
// sums[1][r] += -(gx * c * y) / (d * d), q = y / d, c = min(d, 1), over the rows' entries
// (any entry order).  One wave of blocks, each with shared bins of every row (up to
// kMaxBinRows rows; global atomics beyond), added to the output once per block.
__global__ void __launch_bounds__(kTileThreads) mass_norm_grad_sums_kernel(
    const int64_t* __restrict__ keys, const float* __restrict__ y, const float* __restrict__ gx, int64_t n, FastDiv E,
    int64_t row0, int64_t nrows, const float* __restrict__ d, double* __restrict__ sums, unsigned* err) {
  __shared__ double bins[2][kMaxBinRows];
  const bool binned = nrows <= kMaxBinRows;
  if (binned)
    for (int64_t i = threadIdx.x; i < nrows; i += kTileThreads) { bins[0][i] = 0.0; bins[1][i] = 0.0; }
  __syncthreads();
  for (int64_t i = blockIdx.x * (int64_t)kTileThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kTileThreads) {
    const int64_t r = E.div(keys[i]) - row0;
    if (r < 0 || r >= nrows) {
      raise_flag(err, MKG_DEV_BAD_KEY);
      continue;
    }
    const float yv = y[i];
    if (yv == 0.0f) continue;
    const float dr = d[r];
    const float g = gx[i];
    const float q = __fdiv_rn(yv, dr);
    const float gq = g * fminf(dr, 1.0f);
    // the terms in fp64: the row sums cancel
    const double a0 = (double)g * (double)q;
    const double a1 = -((double)gq * (double)yv) / ((double)dr * (double)dr);
    if (binned) {
      atomicAdd(&bins[0][r], a0);
      atomicAdd(&bins[1][r], a1);
    } else {
      atomicAdd(sums + r, a0);
      atomicAdd(sums + nrows + r, a1);
    }
  }
  if (binned) {
    __syncthreads();
    for (int64_t i = threadIdx.x; i < nrows; i += kTileThreads) {
      if (bins[0][i] != 0.0) atomicAdd(sums + i, bins[0][i]);
      if (bins[1][i] != 0.0) atomicAdd(sums + nrows + i, bins[1][i]);
    }
  }
}

// gy = (gx * c) / d + g_d[row] with g_d = sums[1] + [d <= 1] sums[0] (fp64, rounded once);
// zero where y is zero.
// PUT: gy goes straight into the slab store at the key's slot (the put that precedes the
// transposed walk) instead of into an array.
template <bool PUT>
__global__ void mass_norm_grad_kernel(const int64_t* __restrict__ keys, const float* __restrict__ y,
                                      const float* __restrict__ gx, int64_t n, FastDiv E, int64_t row0,
                                      int64_t nrows, const float* __restrict__ d, const double* __restrict__ sums,
                                      float* __restrict__ gy, Store st, Window win, unsigned* err) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = keys[i];
    const int64_t r = E.div(k) - row0;
    float out = 0.0f;
    if (r >= 0 && r < nrows && y[i] != 0.0f) {
      const float dr = d[r];
      const float gq = gx[i] * fminf(dr, 1.0f);
      const double gd = sums[nrows + r] + (dr <= 1.0f ? sums[r] : 0.0);
      out = static_cast<float>((double)gq / (double)dr + gd);
    }
    if (PUT) {
      const int64_t slot = k < 0 ? -1 : slot_of(win, k, 1);
      if (slot < 0) raise_flag(err, MKG_DEV_BAD_KEY);
      else st.val[slot] = out;
    } else {
      gy[i] = out;
    }
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

// Blocks of `kernel` resident at once on the device.
template <class Kernel>
int resident_grid(Kernel kernel, int threads = kExpandThreads) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  return num_sms() * per_sm;
}

// grid of a grid-stride loop over n items: at most one wave of resident blocks (a partial second
// wave would hold the launch for a whole block's share of the items)
template <class Kernel>
int stride_grid(Kernel kernel, int64_t n, int threads = 256) {
  return grid_for(n, threads, resident_grid(kernel, threads));
}

// The tile lists of a launch from host arrays of device pointers (1..kMaxTiles, none null).
int make_tiles(int32_t ntiles, const int32_t* const* push_ptrs, const mkg_adj_edge* const* pushes, TileLists* tl) {
  MKG_REQUIRE(ntiles >= 1 && ntiles <= kMaxTiles && push_ptrs && pushes,
              "slab: 1 to %d destination tiles expected, got %d", kMaxTiles, (int)ntiles);
  *tl = TileLists{};
  for (int t = 0; t < ntiles; ++t) {
    MKG_REQUIRE(push_ptrs[t] && pushes[t], "slab: null push list of tile %d", t);
    tl->ptr[t] = push_ptrs[t];
    tl->push[t] = reinterpret_cast<const int4*>(pushes[t]);
  }
  for (int t = ntiles; t < kMaxTiles; ++t) {  // never selected (t < count): any valid pointer
    tl->ptr[t] = push_ptrs[0];
    tl->push[t] = reinterpret_cast<const int4*>(pushes[0]);
  }
  tl->count = ntiles;
  return MKG_OK;
}

// Workspace of a walk over `items` work items: chunk offsets [items + 1], the work counter, the
// scan's temporary storage.
int build_chunks(const TileLists& tl, int identity, const int64_t* keys, int64_t nnz, const mkg_slab_window& win,
                 void* ws, size_t ws_bytes, int64_t** chunk_ptr, unsigned long long** next, unsigned* err,
                 cudaStream_t st) {
  const int64_t items = nnz * tl.count;
  int64_t* cp = static_cast<int64_t*>(ws);
  auto* counter = reinterpret_cast<unsigned long long*>(static_cast<char*>(ws) + a256(8 * (size_t)(items + 1)));
  void* temp = reinterpret_cast<char*>(counter) + 256;
  size_t tb = chunk_scan_bytes(items);
  MKG_REQUIRE(ws_bytes >= a256(8 * (size_t)(items + 1)) + 256 + tb, "slab: expand workspace too small");
  chunk_count_kernel<<<stride_grid(chunk_count_kernel, items), 256, 0, st>>>(keys, nnz, win.E, win.row0, win.nrows,
                                                                            tl, identity, cp, counter, err);
  MKG_LAUNCHED("chunk_count_kernel");
  MKG_CUDA(cub::DeviceScan::InclusiveSum(temp, tb, cp, cp, (int)(items + 1), st));
  *chunk_ptr = cp;
  *next = counter;
  return MKG_OK;
}

// The chunk walks run one wave of resident blocks that take chunks from the work counter until
// none are left (blocks beyond the resident ones would only start once the counter ran out).
int expand_grid(int64_t nnz) {
  (void)nnz;
  return resident_grid(slab_expand_kernel, kExpandThreads);
}

int expand_backward_grid(int64_t nnz) {
  (void)nnz;
  return resident_grid(slab_expand_backward_kernel, kExpandThreads);
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
  return a256(8 * (size_t)(nnz + 1)) + 256 + a256(chunk_scan_bytes(nnz));
}

MKG_API int mkg_slab_expand_tiles(int32_t ntiles, const int32_t* const* push_ptrs, const mkg_adj_edge* const* pushes,
                                  const int64_t* keys, const float* vals, int64_t nnz, const float* w, int64_t n,
                                  int32_t identity, int32_t agg_mode, const mkg_slab_window* win, void* store,
                                  double* row_sums, void* workspace, size_t workspace_bytes, unsigned* dev_err,
                                  mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(row_sums == nullptr || agg_mode == 0, "slab_expand: row sums belong to the sum hop (agg_mode 0)");
  MKG_REQUIRE(window_ok(win), "slab_expand: bad window");
  MKG_REQUIRE(nnz >= 0 && n >= 1 && n <= INT32_MAX, "slab_expand: bad sizes");
  MKG_REQUIRE(agg_mode == 0 || agg_mode == 1, "slab_expand: agg_mode must be 0 (sum) or 1 (max)");
  MKG_REQUIRE(ntiles >= 1 && ntiles <= kMaxTiles, "slab: 1 to %d destination tiles expected, got %d", kMaxTiles,
              (int)ntiles);
  if (nnz == 0) return MKG_OK;
  TileLists tl;
  int rc = make_tiles(ntiles, push_ptrs, pushes, &tl);
  if (rc) return rc;
  MKG_REQUIRE(keys && vals && w && store && workspace, "slab_expand: null argument");
  MKG_REQUIRE(nnz * ntiles < INT32_MAX, "slab_expand: %lld frontier entries x %d tiles exceed the scan limit",
              (long long)nnz, (int)ntiles);
  int64_t* cp = nullptr;
  unsigned long long* next = nullptr;
  rc = build_chunks(tl, identity, keys, nnz, *win, workspace, workspace_bytes, &cp, &next, dev_err, st);
  if (rc) return rc;
  ExpandArgs a{tl, keys, vals, nnz, cp, next, w, n, identity, agg_mode, make_window(*win), dev_err, row_sums};
  slab_expand_kernel<<<expand_grid(nnz), kExpandThreads, 0, st>>>(a, make_store(store, win->nrows * win->extent));
  MKG_LAUNCHED("slab_expand_kernel");
  return MKG_OK;
}

MKG_API int mkg_slab_expand(const int32_t* push_ptr, const mkg_adj_edge* push, const int64_t* keys, const float* vals,
                            int64_t nnz, const float* w, int64_t n, int32_t identity, int32_t agg_mode,
                            const mkg_slab_window* win, void* store, double* row_sums, void* workspace,
                            size_t workspace_bytes, unsigned* dev_err, mkg_stream stream) {
  return mkg_slab_expand_tiles(1, &push_ptr, &push, keys, vals, nnz, w, n, identity, agg_mode, win, store, row_sums,
                               workspace, workspace_bytes, dev_err, stream);
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

namespace mkg {
namespace {
int slab_emit_impl(const mkg_slab_window* win, void* store, const void* workspace, size_t workspace_bytes,
                   int64_t count, int64_t* keys_out, float* vals_out, const GatherNorm* nm, cudaStream_t st) {
  MKG_REQUIRE(window_ok(win) && store && workspace, "slab_emit: bad argument");
  MKG_REQUIRE(count >= 0 && (count == 0 || (keys_out && vals_out)), "slab_emit: bad output");
  const int64_t slots = win->nrows * win->extent;
  const int64_t words = bitmap_words(slots), nblk = collect_blocks(slots);
  MKG_REQUIRE(workspace_bytes >= mkg_slab_collect_workspace_bytes(slots), "slab_emit: workspace too small");
  const Store s = make_store(store, slots);
  slab_emit_kernel<<<(unsigned)nblk, kTileThreads, 0, st>>>(s, make_window(*win), words,
                                                            static_cast<const int64_t*>(workspace), count, keys_out);
  MKG_LAUNCHED("slab_emit_kernel");
  if (count > 0) {
    const int64_t per = (int64_t)kTileThreads * kGatherItems;
    const int gblocks = grid_for(count, (int)per, persistent_blocks(16));
    if (nm)
      slab_gather_kernel<true><<<(unsigned)gblocks, kTileThreads, 0, st>>>(s, make_window(*win), keys_out, count,
                                                                           vals_out, *nm);
    else
      slab_gather_kernel<false><<<(unsigned)gblocks, kTileThreads, 0, st>>>(s, make_window(*win), keys_out, count,
                                                                            vals_out, GatherNorm{});
    MKG_LAUNCHED("slab_gather_kernel");
  }
  return MKG_OK;
}
}  // namespace
}  // namespace mkg

MKG_API int mkg_slab_emit(const mkg_slab_window* win, void* store, const void* workspace, size_t workspace_bytes,
                          int64_t count, int64_t* keys_out, float* vals_out, mkg_stream stream) {
  return slab_emit_impl(win, store, workspace, workspace_bytes, count, keys_out, vals_out, nullptr,
                        reinterpret_cast<cudaStream_t>(stream));
}

MKG_API int mkg_slab_emit_normalized(const mkg_slab_window* win, void* store, const void* workspace,
                                     size_t workspace_bytes, int64_t count, const float* row_sums, float threshold,
                                     int64_t* keys_out, float* y_out, float* x_out, int64_t* dropped,
                                     mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(dropped && row_sums && (count == 0 || x_out), "slab_emit_normalized: null argument");
  MKG_CUDA(cudaMemsetAsync(dropped, 0, sizeof(int64_t), st));
  const GatherNorm nm{row_sums, threshold, x_out, reinterpret_cast<unsigned long long*>(dropped)};
  return slab_emit_impl(win, store, workspace, workspace_bytes, count, keys_out, y_out, &nm, st);
}

MKG_API int mkg_slab_put(const mkg_slab_window* win, void* store, const int64_t* keys, const float* vals, int64_t nnz,
                         int64_t row_div, int32_t mode, unsigned* dev_err, mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(window_ok(win) && store && row_div >= 1 && (mode & ~MKG_SLAB_SKIP_OUTSIDE) >= 0 &&
                  (mode & ~MKG_SLAB_SKIP_OUTSIDE) <= 2 && nnz >= 0,
              "slab_put: bad argument");
  if (nnz == 0) return MKG_OK;
  MKG_REQUIRE(keys && vals, "slab_put: null argument");
  slab_put_kernel<<<stride_grid(slab_put_kernel, nnz), 256, 0, st>>>(
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
  slab_take_kernel<<<stride_grid(slab_take_kernel, nnz), 256, 0, st>>>(
      make_store(store, win->nrows * win->extent), make_window(*win), keys, nnz, row_div, out, clear, dev_err);
  MKG_LAUNCHED("slab_take_kernel");
  return MKG_OK;
}

MKG_API int mkg_slab_expand_backward_tiles(int32_t ntiles, const int32_t* const* push_ptrs,
                                           const mkg_adj_edge* const* pushes, const int64_t* keys, const float* vals,
                                           int64_t nnz, const float* w, int64_t n, int32_t identity,
                                           const mkg_slab_window* win, const void* store, const mkg_edge_factor* ef,
                                           int64_t num_facts, double* grad_sp, double* grad_w, float* grad_edge,
                                           void* workspace, size_t workspace_bytes, unsigned* dev_err,
                                           mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(window_ok(win), "slab_expand_backward: bad window");
  MKG_REQUIRE(nnz >= 0 && n >= 1 && n <= INT32_MAX, "slab_expand_backward: bad sizes");
  MKG_REQUIRE(ntiles >= 1 && ntiles <= kMaxTiles, "slab: 1 to %d destination tiles expected, got %d", kMaxTiles,
              (int)ntiles);
  if (nnz == 0) return MKG_OK;
  TileLists tl;
  int rc = make_tiles(ntiles, push_ptrs, pushes, &tl);
  if (rc) return rc;
  MKG_REQUIRE(keys && vals && w && store && ef && grad_sp && grad_w && workspace,
              "slab_expand_backward: null argument");
  MKG_REQUIRE(nnz * ntiles < INT32_MAX, "slab_expand_backward: frontier too large");
  int64_t* cp = nullptr;
  unsigned long long* next = nullptr;
  rc = build_chunks(tl, identity, keys, nnz, *win, workspace, workspace_bytes, &cp, &next, dev_err, st);
  if (rc) return rc;
  ExpandArgs a{tl, keys, vals, nnz, cp, next, w, n, identity, 0, make_window(*win), dev_err, nullptr};
  slab_expand_backward_kernel<<<expand_backward_grid(nnz), kExpandThreads, 0, st>>>(
      a, static_cast<const float*>(store), make_factor(*ef), num_facts, grad_sp, grad_w, grad_edge);
  MKG_LAUNCHED("slab_expand_backward_kernel");
  return MKG_OK;
}

MKG_API int mkg_slab_expand_backward(const int32_t* push_ptr, const mkg_adj_edge* push, const int64_t* keys,
                                     const float* vals, int64_t nnz, const float* w, int64_t n, int32_t identity,
                                     const mkg_slab_window* win, const void* store, const mkg_edge_factor* ef,
                                     int64_t num_facts, double* grad_sp, double* grad_w, float* grad_edge,
                                     void* workspace, size_t workspace_bytes, unsigned* dev_err, mkg_stream stream) {
  return mkg_slab_expand_backward_tiles(1, &push_ptr, &push, keys, vals, nnz, w, n, identity, win, store, ef,
                                        num_facts, grad_sp, grad_w, grad_edge, workspace, workspace_bytes, dev_err,
                                        stream);
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

MKG_API int mkg_mass_normalize(const int64_t* keys, const float* y, int64_t n, int64_t E, int64_t row0, int64_t nrows,
                               const float* row_sums, float threshold, float* x, int64_t* dropped, unsigned* dev_err,
                               mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(E > 0 && nrows > 0 && row0 >= 0 && n >= 0 && dropped, "mass_normalize: bad argument");
  MKG_CUDA(cudaMemsetAsync(dropped, 0, sizeof(int64_t), st));
  if (n == 0) return MKG_OK;
  MKG_REQUIRE(keys && y && row_sums && x, "mass_normalize: null argument");
  mass_norm_kernel<<<stride_grid(mass_norm_kernel, n), 256, 0, st>>>(
      keys, y, n, FastDiv::of(E), row0, nrows, row_sums, threshold, x, reinterpret_cast<unsigned long long*>(dropped), dev_err);
  MKG_LAUNCHED("mass_norm_kernel");
  return MKG_OK;
}

MKG_API int mkg_mass_normalize_grad_sums(const int64_t* keys, const float* y, const float* gx, int64_t n, int64_t E,
                                         int64_t row0, int64_t nrows, const float* row_sums, double* sums,
                                         unsigned* dev_err, mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(E > 0 && nrows > 0 && row0 >= 0 && n >= 0, "mass_normalize_grad_sums: bad sizes");
  if (n == 0) return MKG_OK;
  MKG_REQUIRE(keys && y && gx && row_sums && sums, "mass_normalize_grad_sums: null argument");
  const int blocks = stride_grid(mass_norm_grad_sums_kernel, n, kTileThreads);
  mass_norm_grad_sums_kernel<<<(unsigned)blocks, kTileThreads, 0, st>>>(keys, y, gx, n, FastDiv::of(E), row0, nrows, row_sums,
                                                                         sums, dev_err);
  MKG_LAUNCHED("mass_norm_grad_sums_kernel");
  return MKG_OK;
}

MKG_API int mkg_mass_normalize_grad(const int64_t* keys, const float* y, const float* gx, int64_t n, int64_t E,
                                    int64_t row0, int64_t nrows, const float* row_sums, const double* sums, float* gy,
                                    mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(E > 0 && nrows > 0 && row0 >= 0 && n >= 0, "mass_normalize_grad: bad sizes");
  if (n == 0) return MKG_OK;
  MKG_REQUIRE(keys && y && gx && row_sums && sums && gy, "mass_normalize_grad: null argument");
  mass_norm_grad_kernel<false><<<stride_grid(mass_norm_grad_kernel<false>, n), 256, 0, st>>>(
      keys, y, gx, n, FastDiv::of(E), row0, nrows, row_sums, sums, gy, Store{}, Window{}, nullptr);
  MKG_LAUNCHED("mass_norm_grad_kernel");
  return MKG_OK;
}

MKG_API int mkg_mass_normalize_grad_put(const int64_t* keys, const float* y, const float* gx, int64_t n, int64_t E,
                                        int64_t row0, int64_t nrows, const float* row_sums, const double* sums,
                                        const mkg_slab_window* win, void* store, unsigned* dev_err,
                                        mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(E > 0 && nrows > 0 && row0 >= 0 && n >= 0, "mass_normalize_grad_put: bad sizes");
  MKG_REQUIRE(window_ok(win) && win->E == E, "mass_normalize_grad_put: bad window");
  if (n == 0) return MKG_OK;
  MKG_REQUIRE(keys && y && gx && row_sums && sums && store, "mass_normalize_grad_put: null argument");
  mass_norm_grad_kernel<true><<<stride_grid(mass_norm_grad_kernel<true>, n), 256, 0, st>>>(
      keys, y, gx, n, FastDiv::of(E), row0, nrows, row_sums, sums, nullptr, make_store(store, win->nrows * win->extent),
      make_window(*win), dev_err);
  MKG_LAUNCHED("mass_norm_grad_kernel");
  return MKG_OK;
}

MKG_API int mkg_f64_to_f32(const double* in, int64_t n, float* out, mkg_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MKG_REQUIRE(n >= 0 && (n == 0 || (in && out)), "f64_to_f32: bad argument");
  if (n == 0) return MKG_OK;
  f64_to_f32_kernel<<<stride_grid(f64_to_f32_kernel, n), 256, 0, st>>>(in, n, out);
  MKG_LAUNCHED("f64_to_f32_kernel");
  return MKG_OK;
}
