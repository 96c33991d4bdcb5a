// The fused hop loop on a dense entity-major state (B200, sm_100a).
//
// State X_h is [E][BLP] fp32 (row = entity, column = b*L + l, BLP = B*L rounded up to 4),
// so one entity's frontier across every (query, rule) is a contiguous 128-bit-loadable row.
// A hop is a pull over the merged neighbour list (every message that can reach a row):
//
//   Y[d][c] = X[d][c] * w[n-1][c] + sum_{(s, ch, m) in pull(d)} (X[s][c] * w[ch][c]) * m
//
// which fuses the op's three outputs and sum_sparse3d_concat; the column sums of Y give the
// normalize_sparse3d denominators.  Rows are cut into tasks of at most kSeg edges (a row
// longer than that becomes several tasks that add into the row with fp32 atomics), so hub
// rows never serialise one warp.  Warps take tasks from a queue; each block works on one
// 128-column chunk and keeps the chunk of the rule weights (and, backward, of their
// gradient) in shared memory.  The backward is the same walk over the push list.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cub/cub.cuh>

#include "mkg_common.cuh"

namespace mkg {


constexpr int kChunk = 128;      // columns per block (32 lanes x float4)
constexpr int kFwdWarps = 8;
constexpr int kBwdWarps = 8;
constexpr int kTaskFirst = 1;    // task holds the row's first edges (adds the identity term)
constexpr int kTaskPartial = 2;  // row split over several tasks: accumulate with atomics
constexpr int kBatch = 4;        // backward: edges whose dY rows are loaded together (4 x 16 B per lane)
constexpr int kGrab = 4;         // tasks per queue atomic
constexpr int kQueueStride = 32; // ints between two queue counters

struct ProofDims {
  int64_t B, L, E, R, n, hops, BL, BLP, nch;
  int64_t cap;      // edge cap of the capped loop, -1: uncapped
  int64_t ngroups;  // rows of the per-hop take table (capped loop)
  int64_t tblp;     // take-table row stride: BLP rounded up to 256 columns
};

inline ProofDims proof_dims(const mkg_proof_params& p) {
  ProofDims d;
  d.B = p.B; d.L = p.L; d.E = p.E; d.R = p.R; d.n = 2 * p.R + 1; d.hops = p.hops;
  d.BL = p.B * p.L;
  d.BLP = (d.BL + 3) / 4 * 4;
  d.nch = (d.BLP + kChunk - 1) / kChunk;
  const bool capped = p.topk_edges < (int64_t(1) << 60) && p.cap_index != nullptr;
  d.cap = capped ? p.topk_edges : -1;
  d.ngroups = capped ? p.cap_index->num_groups : 0;
  d.tblp = (d.BLP + 255) / 256 * 256;
  return d;
}

namespace {

size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

struct ProofLayout {
  size_t wt, x, y, d, act, yact, dxa, dxb, dy, s, dwt, queue, msgs, take, total;
};

ProofLayout proof_layout(const ProofDims& q) {
  ProofLayout L{};
  size_t o = 0;
  const size_t slab = 4 * (size_t)q.E * q.BLP;
  L.wt = o; o += a256(4 * (size_t)q.hops * q.n * q.BLP);
  L.x = o; o += a256(slab) * (q.hops + 1);
  L.y = o; o += a256(slab) * q.hops;
  L.d = o; o += a256(4 * (size_t)q.hops * q.BLP);
  L.act = o; o += a256((size_t)(q.hops + 1) * q.E * q.nch);
  L.yact = o; o += a256((size_t)q.hops * q.E * q.nch);
  L.dxa = o; o += a256(slab);
  L.dxb = o; o += a256(slab);
  L.dy = o; o += a256(slab);
  L.s = o; o += a256(8 * (size_t)q.hops * q.BLP);  // fp64: S sums dX Y terms of both signs
  L.dwt = o; o += a256(8 * (size_t)q.n * q.BLP);  // fp64 accumulator
  L.queue = o; o += a256(4 * (size_t)(2 * q.hops * q.nch * kQueueStride));
  L.msgs = o; o += a256(8 * (size_t)(q.hops + 1));
  L.take = o; o += a256((size_t)q.hops * q.ngroups * q.tblp);
  L.total = o;
  return L;
}

struct Slab {
  char* base;
  ProofLayout lay;
  ProofDims q;
  float* wt(int64_t h) const { return reinterpret_cast<float*>(base + lay.wt) + h * q.n * q.BLP; }
  float* x(int64_t h) const { return reinterpret_cast<float*>(base + lay.x + a256(4 * (size_t)q.E * q.BLP) * h); }
  float* y(int64_t h) const { return reinterpret_cast<float*>(base + lay.y + a256(4 * (size_t)q.E * q.BLP) * h); }
  float* d(int64_t h) const { return reinterpret_cast<float*>(base + lay.d) + h * q.BLP; }
  uint8_t* act(int64_t h) const { return reinterpret_cast<uint8_t*>(base + lay.act) + h * q.E * q.nch; }
  // non-zero pattern of Y_h per (row, chunk): where the backward's dY_h can be non-zero
  uint8_t* yact(int64_t h) const { return reinterpret_cast<uint8_t*>(base + lay.yact) + h * q.E * q.nch; }
  float* dxa() const { return reinterpret_cast<float*>(base + lay.dxa); }
  float* dxb() const { return reinterpret_cast<float*>(base + lay.dxb); }
  float* dy() const { return reinterpret_cast<float*>(base + lay.dy); }
  double* s(int64_t h) const { return reinterpret_cast<double*>(base + lay.s) + h * q.BLP; }
  double* dwt() const { return reinterpret_cast<double*>(base + lay.dwt); }
  int32_t* queue() const { return reinterpret_cast<int32_t*>(base + lay.queue); }
  int64_t* msgs() const { return reinterpret_cast<int64_t*>(base + lay.msgs); }
  // edge-cap take table of hop h: [ngroups][tblp] edges taken per (capped group, column), columns
  // permuted within each 256-column tile (take_offset)
  uint8_t* take(int64_t h) const { return reinterpret_cast<uint8_t*>(base + lay.take) + h * q.ngroups * q.tblp; }
};

// ------------------------------------------------------------------ setup kernels
// Wt[h][ch][c] = w_hops[h][b][l][ch] for c = b*L + l (zero in the padding columns).
__global__ void transpose_w_kernel(const float* __restrict__ w, ProofDims q, float* __restrict__ wt) {
  const int64_t total = q.hops * q.n * q.BLP;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t c = i % q.BLP, rest = i / q.BLP, ch = rest % q.n, h = rest / q.n;
    wt[i] = c < q.BL ? w[(h * q.BL + c) * q.n + ch] : 0.0f;
  }
}

// grad_w_hops[h][b][l][ch] = dWt[ch][b*L + l], rounded once from the fp64 accumulator; dWt is
// cleared behind the read for the next lower hop (its padding columns receive nothing and stay
// zero).
__global__ void untranspose_dw_kernel(double* __restrict__ dwt, ProofDims q, int64_t h, float* __restrict__ gw) {
  const int64_t total = q.BL * q.n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t ch = i % q.n, c = i / q.n;
    gw[h * total + i] = static_cast<float>(dwt[ch * q.BLP + c]);
    dwt[ch * q.BLP + c] = 0.0;
  }
}

// Start of a forward, one launch for what must be zero before it: the activity flags and Y
// marks of every hop (bytes [flags, flags + nflags)), the column sums, the forward's task-queue
// counters, the message counts, the head rows of X_0 (the only rows of X_0 the hop-0 pull
// reads, as act_0 is set only there; both halves of a 256-column pair are zeroed with the row)
// and, for every hop, the rows of Y_h that several pull tasks add into.
__global__ void forward_setup_kernel(const int64_t* __restrict__ heads, const int4* __restrict__ tasks, int64_t ntasks,
                                     ProofDims q, uint8_t* __restrict__ flags, int64_t nflags,
                                     float* __restrict__ y0, int64_t y_stride, float* __restrict__ x0,
                                     float* __restrict__ d, int32_t* __restrict__ queue, int64_t nqueue,
                                     int64_t* __restrict__ msgs) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
  for (int64_t i = tid; i < nflags / 16; i += nthreads) reinterpret_cast<uint4*>(flags)[i] = z4;
  for (int64_t i = nflags / 16 * 16 + tid; i < nflags; i += nthreads) flags[i] = 0;
  for (int64_t i = tid; i < q.hops * q.BLP; i += nthreads) d[i] = 0.0f;
  for (int64_t i = tid; i < nqueue; i += nthreads) queue[i] = 0;
  for (int64_t i = tid; i <= q.hops; i += nthreads) msgs[i] = 0;
  const int64_t row4 = q.BLP / 4;  // BLP is a multiple of 4
  for (int64_t i = tid; i < q.B * row4; i += nthreads) {
    const int64_t e = heads[i / row4];
    if (e >= 0 && e < q.E) reinterpret_cast<uint4*>(x0 + e * q.BLP)[i % row4] = z4;  // bad heads: init_state flags them
  }
  const int lane = threadIdx.x & 31;
  for (int64_t t = tid >> 5; t < ntasks; t += nthreads >> 5) {
    const int4 tk = tasks[t];
    if ((tk.w & (kTaskFirst | kTaskPartial)) != (kTaskFirst | kTaskPartial)) continue;
    for (int64_t h = 0; h < q.hops; ++h) {
      uint4* row = reinterpret_cast<uint4*>(y0 + h * y_stride + (int64_t)tk.x * q.BLP);
      for (int64_t j = lane; j < row4; j += 32) row[j] = z4;
    }
  }
}

// Start of a backward: the edge-score gradient, the S sums of every hop, the backward's
// task-queue counters and dWt.
__global__ void backward_setup_kernel(ProofDims q, float* __restrict__ grad_edge, int64_t num_facts,
                                      double* __restrict__ s, int32_t* __restrict__ queue, int64_t nqueue,
                                      double* __restrict__ dwt) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  if (grad_edge)
    for (int64_t i = tid; i < num_facts; i += nthreads) grad_edge[i] = 0.0f;
  for (int64_t i = tid; i < q.hops * q.BLP; i += nthreads) s[i] = 0.0;
  for (int64_t i = tid; i < nqueue; i += nthreads) queue[i] = 0;
  for (int64_t i = tid; i < q.n * q.BLP; i += nthreads) dwt[i] = 0.0;
}

// One-hot start: X0[head_b][b*L + l] = 1 for every rule l (proof.py:511-523).
__global__ void init_state_kernel(const int64_t* __restrict__ heads, ProofDims q, float* __restrict__ x0,
                                  uint8_t* __restrict__ act0, const int32_t* __restrict__ push_ptr,
                                  const int32_t* __restrict__ capdeg, int64_t* __restrict__ msgs, unsigned* err) {
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < q.BL;
       c += (int64_t)gridDim.x * blockDim.x) {
    int64_t b = c / q.L;
    int64_t e = heads[b];
    if (e < 0 || e >= q.E) { raise_flag(err, MKG_DEV_BAD_ENTRY); continue; }
    x0[e * q.BLP + c] = 1.0f;
    act0[e * q.nch + c / kChunk] = 1;
    atomicAdd(reinterpret_cast<unsigned long long*>(msgs),
              (unsigned long long)(capdeg ? capdeg[e] : push_ptr[e + 1] - push_ptr[e]));
  }
}

__device__ __forceinline__ float4 f4_mul(const float4& a, const float4& b) {
  return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w);
}
__device__ __forceinline__ void f4_max_msg(float4& acc, const float4& x, const float4& w, float m) {
  // message value (x * w) * m exactly as the reference forms it, then max
  acc.x = fmaxf(acc.x, (x.x * w.x) * m);
  acc.y = fmaxf(acc.y, (x.y * w.y) * m);
  acc.z = fmaxf(acc.z, (x.z * w.z) * m);
  acc.w = fmaxf(acc.w, (x.w * w.w) * m);
}
__device__ __forceinline__ int f4_count(const float4& v) {
  return (v.x != 0.f) + (v.y != 0.f) + (v.z != 0.f) + (v.w != 0.f);
}

// Dynamic task queue: a warp takes kGrab consecutive tasks per atomic and requests the
// next group as soon as it starts one, so the atomic's latency overlaps the work.  Each
// counter sits on its own 128-byte line (kQueueStride ints apart).
struct TaskCursor {
  int32_t* counter;
  int64_t ntasks;
  int64_t base;
  int pending;  // lane 0: the next group's first task, not yet broadcast
  int i;
  __device__ __forceinline__ TaskCursor(int32_t* c, int64_t n) : counter(c), ntasks(n), i(0) {
    const int lane = threadIdx.x & 31;
    int b = 0;
    if (lane == 0) b = atomicAdd(counter, kGrab);
    base = __shfl_sync(0xffffffffu, b, 0);
    pending = lane == 0 ? atomicAdd(counter, kGrab) : 0;
  }
  __device__ __forceinline__ bool next(int64_t& t) {
    if (i == kGrab) {
      base = __shfl_sync(0xffffffffu, pending, 0);
      if (base < ntasks && (threadIdx.x & 31) == 0) pending = atomicAdd(counter, kGrab);
      i = 0;
    }
    t = base + i;
    ++i;
    return t < ntasks;
  }
};

// VEC float4 of one lane: columns col0 + 4*lane + 128*v, v < VEC.
template <int VEC>
struct Lanes {
  float4 v[VEC];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int k = 0; k < VEC; ++k) v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
};

// Activity flags are kept per 128-column chunk; a VEC-wide chunk is active if any of its
// VEC sub-chunks is.
template <int VEC>
__device__ __forceinline__ bool active_vec(const uint8_t* __restrict__ act, int64_t row, int64_t chunk, int64_t nch) {
  bool a = false;
#pragma unroll
  for (int v = 0; v < VEC; ++v)
    if (chunk * VEC + v < nch) a = a || act[row * nch + chunk * VEC + v] != 0;
  return a;
}

template <int VEC>
__device__ __forceinline__ void load_lanes(Lanes<VEC>& out, const float* __restrict__ rowp, int64_t col,
                                           int64_t BLP) {
#pragma unroll
  for (int k = 0; k < VEC; ++k)
    out.v[k] = (col + 128 * k < BLP) ? *reinterpret_cast<const float4*>(rowp + col + 128 * k)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
}

// ------------------------------------------------------------------ edge cap
// Take table of one hop, the edge cap of fastlog.cu:2092-2195, 2273-2298 for every capped
// row (slot) and column c: the row's relation groups are bucketed by their rule weight
// w[channel][c]; the threshold bucket tb is the largest bucket whose groups at or above it
// hold at least cap edges; groups above tb take all their edges, groups below none, groups
// in tb take, in group order, what is left of cap after the groups above.
// take[row of group][c] = edges taken (its first ones in CSR order).  Block = (slot, tile of
// kTakeCols columns), one thread per column; the buckets of up to kTakeGroups groups are
// computed once into shared memory ([group][column] bytes), longer rows re-read the weights.
// The threshold is found with two histogram passes over the groups (16 coarse bins, then the 16
// buckets of the coarse bin that holds it), whatever the range of the buckets.
// Byte offset of column c inside a take-table row.  Within each 256-column tile the 8 columns a
// forward lane covers (c = 4 lane + i and 128 + 4 lane + i, i < 4) are contiguous: lane l's bytes
// are [8 l, 8 l + 8), the first 4 for the lower 128 columns.  A forward lane reads its take bytes
// with one 8-byte load, a backward lane (128-column chunks) with one 4-byte load.
__host__ __device__ __forceinline__ int64_t take_offset(int64_t c) {
  const int64_t w = c & 255;
  return (c - w) + ((w & 127) >> 2) * 8 + (w >> 7) * 4 + (w & 3);
}
// first byte of the 4 take bytes of 128-column chunk `chunk`, lane `lane`
__device__ __forceinline__ int64_t take_lane_offset(int64_t chunk, int lane) {
  return (chunk >> 1) * 256 + lane * 8 + (chunk & 1) * 4;
}

constexpr int kTakeCols = 256;
constexpr int kTakeGroups = 96;
constexpr int kTakeBins = 16;  // the 256 buckets searched as 16 coarse bins of 16 buckets each

// h += n, saturated at 0xffff.  Exact for the searches below: they compare running sums against
// cap <= 255 and stop at the first bin that reaches it, so only bins below cap are ever added up.
__device__ __forceinline__ void add_saturated(uint16_t& h, int n) {
  const int v = h + n;
  h = static_cast<uint16_t>(v < 0xffff ? v : 0xffff);
}

__global__ void __launch_bounds__(kTakeCols) cap_take_kernel(
    DirCSR ori, DirCSR inv, const int32_t* __restrict__ slot_entity, const int32_t* __restrict__ slot_dir,
    const int32_t* __restrict__ slot_group, int64_t num_slots, ProofDims q, const float* __restrict__ wt,
    const uint8_t* __restrict__ act, uint8_t* __restrict__ take, unsigned* err) {
  __shared__ uint8_t bk[kTakeGroups * kTakeCols];     // [group][column] buckets
  __shared__ uint16_t hist[kTakeBins * kTakeCols];    // [bin][column] edges, coarse then fine level
  __shared__ int32_t gcnt[kTakeGroups];               // group edge counts, clamped at 255
  __shared__ int32_t grel[kTakeGroups];
  const int tid = threadIdx.x;
  const int64_t tiles = (q.BLP + kTakeCols - 1) / kTakeCols;
  uint16_t* hcol = hist + tid;  // this column's bins, kTakeCols apart
  for (int64_t blk = blockIdx.x; blk < num_slots * tiles; blk += gridDim.x) {
    const int64_t slot = blk / tiles;
    const int64_t c = (blk % tiles) * kTakeCols + tid;
    const int dir = slot_dir[slot];
    const DirCSR d = dir == 0 ? ori : inv;
    const int64_t e = slot_entity[slot];
    const int64_t g0 = d.group_ptr[e];
    const int G = static_cast<int>(d.group_ptr[e + 1] - g0);
    // only columns the pulls can read: the sending row's chunk holds state (inactive chunks are
    // skipped there)
    const bool col_active = c < q.BLP && act[e * q.nch + c / kChunk] != 0;
    if (!__syncthreads_or(col_active)) continue;  // uniform over the block
    const bool staged = G <= kTakeGroups;
    const float* w = wt + (dir == 0 ? 0 : q.R) * q.BLP + (c < q.BLP ? c : 0);
    // a relation outside [0, R) is flagged and counts as bucket 0
    auto bucket_at = [&](int32_t rel) { return rel < 0 ? 0 : weight_bucket(w[(int64_t)rel * q.BLP]); };
    auto rel_of = [&](int g) -> int32_t {
      const int32_t rel = d.group_rel[g0 + g];
      if (rel < 0 || rel >= q.R) { raise_flag(err, MKG_DEV_BAD_REL); return -1; }
      return rel;
    };
    __syncthreads();  // the previous slot's shared arrays are consumed
    if (staged) {
      for (int g = tid; g < G; g += blockDim.x) {
        const int32_t cnt = d.group_count[g0 + g];
        gcnt[g] = cnt < 255 ? cnt : 255;
        grel[g] = rel_of(g);
      }
    }
    __syncthreads();
    if (!col_active) continue;
    // Counts are clamped at 255: every comparison below is against cap <= 255, and a group
    // counted before the threshold holds fewer than cap edges, so no decision changes.
    auto count = [&](int g) -> int {
      if (staged) return gcnt[g];
      const int32_t cnt = d.group_count[g0 + g];
      return cnt < 255 ? cnt : 255;
    };
    auto bucket = [&](int g) -> int { return staged ? bk[g * kTakeCols + tid] : bucket_at(rel_of(g)); };
    // tb: the largest bucket whose groups at or above it hold >= cap edges (a capped row holds
    // more than cap); above: the edges of the groups above tb.  Coarse level: buckets >> 4.
#pragma unroll
    for (int k = 0; k < kTakeBins; ++k) hcol[k * kTakeCols] = 0;
#pragma unroll 4
    for (int g = 0; g < G; ++g) {
      const int b = staged ? bucket_at(grel[g]) : bucket_at(rel_of(g));
      if (staged) bk[g * kTakeCols + tid] = static_cast<uint8_t>(b);
      add_saturated(hcol[(b >> 4) * kTakeCols], count(g));
    }
    int above = 0, cb = 0;
    for (int k = kTakeBins - 1; k >= 0; --k) {
      const int h = hcol[k * kTakeCols];
      if (above + h >= q.cap || k == 0) { cb = k; break; }
      above += h;
    }
    // fine level: the buckets of coarse bin cb
#pragma unroll
    for (int k = 0; k < kTakeBins; ++k) hcol[k * kTakeCols] = 0;
    for (int g = 0; g < G; ++g) {
      const int b = bucket(g);
      if ((b >> 4) == cb) add_saturated(hcol[(b & 15) * kTakeCols], count(g));
    }
    int tb = cb * kTakeBins;
    for (int k = kTakeBins - 1; k >= 0; --k) {
      const int h = hcol[k * kTakeCols];
      if (above + h >= q.cap || k == 0) { tb = cb * kTakeBins + k; break; }
      above += h;
    }
    const int remain = static_cast<int>(q.cap) - above;
    int prior = 0;
    uint8_t* out = take + (int64_t)slot_group[slot] * q.tblp + take_offset(c);
    for (int g = 0; g < G; ++g, out += q.tblp) {
      const int b = bucket(g);
      const int cnt = count(g);
      int t = b > tb ? cnt : 0;
      if (b == tb) {
        t = remain - prior;
        t = t < 0 ? 0 : (t > cnt ? cnt : t);
        prior += cnt;
      }
      *out = static_cast<uint8_t>(t);
    }
  }
}

// Keeps the columns of v whose take byte in t4 exceeds the record's position in its group
// (one SIMD byte compare; a position >= 255 is never taken since takes are at most 255).
__device__ __forceinline__ float4 cap_masked(float4 v, unsigned t4, int pos) {
  const unsigned p = pos < 255 ? static_cast<unsigned>(pos) : 255u;
  const unsigned m = __vcmpgtu4(t4, p * 0x01010101u);  // 0xff in every byte where take > pos
  v.x = __int_as_float(__float_as_int(v.x) & static_cast<int>(__byte_perm(m, 0, 0x0000)));
  v.y = __int_as_float(__float_as_int(v.y) & static_cast<int>(__byte_perm(m, 0, 0x1111)));
  v.z = __int_as_float(__float_as_int(v.z) & static_cast<int>(__byte_perm(m, 0, 0x2222)));
  v.w = __int_as_float(__float_as_int(v.w) & static_cast<int>(__byte_perm(m, 0, 0x3333)));
  return v;
}

// ------------------------------------------------------------------ forward pull
// One warp per task (a segment of <= 64 records of one pull row) and column chunk of
// 128*VEC columns.  Per batch of 32 records, the records whose source row is active in this
// chunk are compacted into shared memory (one ballot), then walked four at a time.
// MAX = false: sum aggregation.  Records of a row come grouped by channel, so m * X[src]
// is summed per channel run and multiplied by the run's rule weights once (fp32 order
// differs from the per-message products; the sum is within tolerance).  Column sums of
// the output feed normalize_sparse3d, and every (row, 128-column chunk) this warp adds a
// non-zero value to is marked in yhint (zeroed before the forward), so that the normalisation
// reads only those chunks.
// MAX = true: max of the exact message values (X[src] * w[ch]) * m (sparse3d_max over the
// op's ind / ori / inv outputs), rule weights read per record.
template <bool MAX, int VEC, bool CAP>
__global__ void __launch_bounds__(kFwdWarps * 32) fwd_pull_kernel(
    const int4* __restrict__ tasks, int64_t ntasks, const mkg_adj_edge* __restrict__ edges, ProofDims q,
    const float* __restrict__ wt, const float* __restrict__ x, const uint8_t* __restrict__ act,
    float* __restrict__ y, float* __restrict__ dsum, uint8_t* __restrict__ yhint, int32_t* __restrict__ queue,
    const int2* __restrict__ rcap, const uint8_t* __restrict__ take, unsigned* err) {
  __shared__ int4 recs[kFwdWarps][32];
  __shared__ int2 rcs[kFwdWarps][CAP ? 32 : 1];  // capped records: (take row, position in group)
  __shared__ float cs[4 * 32 * VEC];  // column partial sums: cs[(v*4 + k)*32 + lane] = column 4*lane + k + 128*v
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t chunk = blockIdx.y;
  const int64_t col0 = chunk * (128 * VEC);
  const int64_t col = col0 + 4 * lane;
  if (!MAX)
    for (int i = threadIdx.x; i < 4 * 32 * VEC; i += blockDim.x) cs[i] = 0.0f;
  __syncthreads();
  Lanes<VEC> csum;
  csum.zero();
  TaskCursor cursor(queue + chunk * kQueueStride, ntasks);
  int64_t t;
  while (cursor.next(t)) {
    const int4 tk = tasks[t];
    const int64_t row = tk.x;
    Lanes<VEC> acc, run;
    acc.zero();
    run.zero();
    if ((tk.w & kTaskFirst) && active_vec<VEC>(act, row, chunk, q.nch)) {
      Lanes<VEC> xr, wi;
      load_lanes(xr, x + row * q.BLP, col, q.BLP);
      load_lanes(wi, wt + (q.n - 1) * q.BLP, col, q.BLP);
#pragma unroll
      for (int k = 0; k < VEC; ++k) acc.v[k] = f4_mul(xr.v[k], wi.v[k]);
    }
    int cur = -1;
    for (int base = tk.y; base < tk.z; base += 32) {
      const int cnt = min(32, tk.z - base);
      int4 rec = make_int4(0, 0, 0, 0);
      int2 rc = make_int2(-1, 0);
      bool live = false;
      if (lane < cnt) {
        rec = reinterpret_cast<const int4*>(edges)[base + lane];
        if (CAP) rc = rcap[base + lane];
        if (rec.x < 0 || rec.x >= q.E || rec.y < 0 || rec.y >= q.n - 1) raise_flag(err, MKG_DEV_BAD_COL);
        else if (CAP && rc.x >= q.ngroups) raise_flag(err, MKG_DEV_BAD_ENTRY);
        else live = active_vec<VEC>(act, rec.x, chunk, q.nch);
      }
      const unsigned mask = __ballot_sync(0xffffffffu, live);
      const int nact = __popc(mask);
      if (live) {
        const int slot = __popc(mask & ((1u << lane) - 1u));
        recs[warp][slot] = rec;
        if (CAP) rcs[warp][slot] = rc;
      }
      __syncwarp();
      for (int k0 = 0; k0 < nact; k0 += 4) {
        int4 r[4];
        Lanes<VEC> xv[4];
        unsigned tw[4][VEC];  // take words, loaded with the X rows (capped loop)
        int tp[4];            // positions inside the capped groups
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          r[u] = (k0 + u < nact) ? recs[warp][k0 + u] : make_int4(0, -1, 0, 0);
          if (r[u].y >= 0) {
            load_lanes(xv[u], x + (int64_t)r[u].x * q.BLP, col, q.BLP);
            if (CAP) {
              const int2 cr = rcs[warp][k0 + u];
              tp[u] = cr.x >= 0 ? cr.y : -1;  // -1: a record of an uncapped row
              const uint8_t* tr = take + (int64_t)(cr.x >= 0 ? cr.x : 0) * q.tblp;
              if (VEC == 2) {
                const uint2 t8 = cr.x >= 0 ? __ldg(reinterpret_cast<const uint2*>(tr + chunk * 256 + lane * 8))
                                           : make_uint2(0xFFFFFFFFu, 0xFFFFFFFFu);
                tw[u][0] = t8.x;
                tw[u][VEC - 1] = t8.y;
              } else {
                tw[u][0] = cr.x >= 0 ? __ldg(reinterpret_cast<const unsigned*>(tr + take_lane_offset(chunk, lane)))
                                     : 0xFFFFFFFFu;
              }
            }
          }
        }

#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (r[u].y < 0) continue;
          if (CAP && tp[u] >= 0) {  // uniform over the warp (one record)
#pragma unroll
            for (int k = 0; k < VEC; ++k) xv[u].v[k] = cap_masked(xv[u].v[k], tw[u][k], tp[u]);
          }
          const float m = __int_as_float(r[u].w);
          if (MAX) {
            Lanes<VEC> wv;
            load_lanes(wv, wt + (int64_t)r[u].y * q.BLP, col, q.BLP);
#pragma unroll
            for (int k = 0; k < VEC; ++k) f4_max_msg(acc.v[k], xv[u].v[k], wv.v[k], m);
          } else {
            if (r[u].y != cur) {
              if (cur >= 0) {
                Lanes<VEC> wc;
                load_lanes(wc, wt + (int64_t)cur * q.BLP, col, q.BLP);
#pragma unroll
                for (int k = 0; k < VEC; ++k) {
                  acc.v[k].x = fmaf(run.v[k].x, wc.v[k].x, acc.v[k].x);
                  acc.v[k].y = fmaf(run.v[k].y, wc.v[k].y, acc.v[k].y);
                  acc.v[k].z = fmaf(run.v[k].z, wc.v[k].z, acc.v[k].z);
                  acc.v[k].w = fmaf(run.v[k].w, wc.v[k].w, acc.v[k].w);
                }
                run.zero();
              }
              cur = r[u].y;
            }
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
              run.v[k].x = fmaf(xv[u].v[k].x, m, run.v[k].x);
              run.v[k].y = fmaf(xv[u].v[k].y, m, run.v[k].y);
              run.v[k].z = fmaf(xv[u].v[k].z, m, run.v[k].z);
              run.v[k].w = fmaf(xv[u].v[k].w, m, run.v[k].w);
            }
          }
        }
      }
      __syncwarp();
    }
    if (!MAX && cur >= 0) {
      Lanes<VEC> wc;
      load_lanes(wc, wt + (int64_t)cur * q.BLP, col, q.BLP);
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        acc.v[k].x = fmaf(run.v[k].x, wc.v[k].x, acc.v[k].x);
        acc.v[k].y = fmaf(run.v[k].y, wc.v[k].y, acc.v[k].y);
        acc.v[k].z = fmaf(run.v[k].z, wc.v[k].z, acc.v[k].z);
        acc.v[k].w = fmaf(run.v[k].w, wc.v[k].w, acc.v[k].w);
      }
    }
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      const int64_t c = col + 128 * k;
      const float4 a = acc.v[k];
      if (!MAX) {
        const bool nz = c < q.BLP && (a.x != 0.f || a.y != 0.f || a.z != 0.f || a.w != 0.f);
        if (__ballot_sync(0xffffffffu, nz) != 0u && lane == 0) yhint[row * q.nch + (col0 >> 7) + k] = 1;
      }
      if (c >= q.BLP) continue;
      float* yr = y + row * q.BLP + c;
      if (tk.w & kTaskPartial) {
        if (MAX) {
          atomicMax(reinterpret_cast<int*>(yr) + 0, __float_as_int(a.x));
          atomicMax(reinterpret_cast<int*>(yr) + 1, __float_as_int(a.y));
          atomicMax(reinterpret_cast<int*>(yr) + 2, __float_as_int(a.z));
          atomicMax(reinterpret_cast<int*>(yr) + 3, __float_as_int(a.w));
        } else {
          atomicAdd(yr + 0, a.x); atomicAdd(yr + 1, a.y);
          atomicAdd(yr + 2, a.z); atomicAdd(yr + 3, a.w);
        }
      } else {
        *reinterpret_cast<float4*>(yr) = a;
      }
      if (!MAX) { csum.v[k].x += a.x; csum.v[k].y += a.y; csum.v[k].z += a.z; csum.v[k].w += a.w; }
    }
  }
  if (!MAX) {
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      atomicAdd(cs + (k * 4 + 0) * 32 + lane, csum.v[k].x);
      atomicAdd(cs + (k * 4 + 1) * 32 + lane, csum.v[k].y);
      atomicAdd(cs + (k * 4 + 2) * 32 + lane, csum.v[k].z);
      atomicAdd(cs + (k * 4 + 3) * 32 + lane, csum.v[k].w);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 4 * 32 * VEC; i += blockDim.x) {
      const int l = i % 32, kk = (i / 32) % 4, v = i / 128;
      const int64_t c = col0 + 4 * l + kk + 128 * v;
      if (c < q.BLP && cs[i] != 0.0f) atomicAdd(dsum + c, cs[i]);
    }
  }
}

// normalize_sparse3d(.., 0, "mass") (drum.py:31-51) on the dense state:
// x = (y / d) * min(d, 1) where y != 0; optional threshold; activity flags and the
// message count of the next hop (present entries x push degree, or x the capped degree).
// yact holds on entry the forward pull's marks (chunks it added a non-zero value to; Y is zero
// in the others) and on exit the exact flags of Y's non-zero chunks.  Unmarked chunks are not
// read and get zeros in X, except where nothing reads them: the pulls read X only in chunks
// whose 256-column pair (chunks 2j, 2j + 1) holds an active chunk, so a chunk whose pair has no
// mark is skipped, on every hop but the last (read whole).  A warp takes kNormTasks (row,
// chunk) tasks at a time, loads first.
constexpr int kNormTasks = 4;

__global__ void __launch_bounds__(256, 4) normalize_mass_kernel(
    const float* __restrict__ y, const float* __restrict__ dsum, ProofDims q, float threshold, bool last_hop,
    float* __restrict__ x, uint8_t* __restrict__ act, uint8_t* __restrict__ yact,
    const int32_t* __restrict__ push_ptr, const int32_t* __restrict__ capdeg, int64_t* __restrict__ msgs) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t total = q.E * q.nch;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  long long local_msgs = 0;
  for (int64_t t0 = warp0 * kNormTasks; t0 < total; t0 += nwarps * kNormTasks) {
    const int64_t row0 = t0 / q.nch, chunk0 = t0 % q.nch;
    bool marked[kNormTasks], pair[kNormTasks];  // uniform over the warp
    float4 v[kNormTasks];
    {
      int64_t row = row0, chunk = chunk0;
#pragma unroll
      for (int u = 0; u < kNormTasks; ++u) {
        const int64_t col = chunk * kChunk + 4 * lane;
        const bool in = t0 + u < total;
        marked[u] = in && yact[t0 + u] != 0;
        pair[u] = marked[u] || (in && (chunk ^ 1) < q.nch && yact[row * q.nch + (chunk ^ 1)] != 0);
        v[u] = (marked[u] && col < q.BLP) ? *reinterpret_cast<const float4*>(y + row * q.BLP + col) : zero;
        if (++chunk == q.nch) { chunk = 0; ++row; }
      }
    }
    int64_t row = row0, chunk = chunk0;
#pragma unroll
    for (int u = 0; u < kNormTasks; ++u) {
      if (t0 + u >= total) break;  // uniform over the warp
      const int64_t col = chunk * kChunk + 4 * lane;
      float4 o = zero;
      bool ynz = false;
      if (marked[u] && col < q.BLP) {
        const float4 vv = v[u];
        ynz = vv.x != 0.f || vv.y != 0.f || vv.z != 0.f || vv.w != 0.f;
        const float4 d = *reinterpret_cast<const float4*>(dsum + col);
        float vi[4] = {vv.x, vv.y, vv.z, vv.w}, di[4] = {d.x, d.y, d.z, d.w}, oi[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float r = 0.0f;
          if (vi[k] != 0.0f) {
            r = __fdiv_rn(vi[k], di[k]) * fminf(di[k], 1.0f);
            if (threshold > 0.0f && r < threshold) r = 0.0f;
          }
          oi[k] = r;
        }
        o = make_float4(oi[0], oi[1], oi[2], oi[3]);
        *reinterpret_cast<float4*>(x + row * q.BLP + col) = o;
      } else if ((pair[u] || last_hop) && col < q.BLP) {
        *reinterpret_cast<float4*>(x + row * q.BLP + col) = zero;
      }
      const int nz = f4_count(o);
      const unsigned any = __ballot_sync(0xffffffffu, nz > 0);
      const unsigned yany = __ballot_sync(0xffffffffu, ynz);
      int tot = nz;
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, s);
      if (lane == 0) {
        act[row * q.nch + chunk] = any ? 1 : 0;
        if (marked[u]) yact[row * q.nch + chunk] = yany ? 1 : 0;
        if (tot) local_msgs += (long long)tot * (capdeg ? capdeg[row] : push_ptr[row + 1] - push_ptr[row]);
      }
      if (++chunk == q.nch) { chunk = 0; ++row; }
    }
  }
  if (lane == 0 && local_msgs) atomicAdd(reinterpret_cast<unsigned long long*>(msgs), (unsigned long long)local_msgs);
}

// norm_sp_3d (src/model_mmDRUM_kernel_sp.py:39-52) column sums, bit-exact: one thread per
// column adds the column top to bottom in fp32 (the reference's index_put_ order), then
// clamps at 1e-7.
// A block owns 32 columns.  Lane 0 of warp 1 streams 64-row x 32-column tiles of Y into a
// ring of kColsumStages shared-memory slots with 2D TMA tensor copies (one instruction per
// 8 KB tile, each completing a "full" mbarrier); warp 0 waits for each tile in order, adds
// it row by row (one lane per column, so the fp32 order stays strictly top to bottom) and
// frees the slot on its "empty" mbarrier.  Every wait is bounded: one that gives up sets
// MKG_DEV_TIMEOUT and a shared stop flag, after which the producer issues no further copy
// and the consumer leaves its loop; before the block exits, one thread waits (bounded again)
// on the full barrier of every tile that was issued but not consumed, so no copy into this
// block's shared memory is left in flight.
constexpr int kColsumRows = 64;
constexpr int kColsumStages = 5;  // 5 x 8 KB ring (static shared memory stays under 48 KB)
constexpr uint32_t kWaitPolls = 1u << 22;

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 2D tiled TMA load of box (x = column, y = row) of `map` into shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__global__ void __launch_bounds__(64) sequential_colsum_kernel(const __grid_constant__ CUtensorMap ymap, ProofDims q,
                                                               float* __restrict__ d, unsigned* err) {
  __shared__ __align__(128) float buf[kColsumStages][kColsumRows][32];
  __shared__ __align__(8) uint64_t full[kColsumStages];
  __shared__ __align__(8) uint64_t empty[kColsumStages];
  __shared__ int stop;                  // set by whichever side gave up on a wait
  __shared__ long long issued, consumed; // tiles copied in / added up
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c0 = (int64_t)blockIdx.x * 32;
  const int ncols = (int)((q.BLP - c0) < 32 ? (q.BLP - c0) : 32);
  const int64_t ntiles = (q.E + kColsumRows - 1) / kColsumRows;
  constexpr uint32_t kTileBytes = kColsumRows * 32 * 4;  // out-of-range rows / columns arrive as zeros
  volatile int* vstop = &stop;
  // bounded wait that also gives up as soon as the other side has stopped
  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
      if (mbar_try_wait(bar, parity)) return true;
      if ((i & 1023u) == 1023u && *vstop) return false;
    }
    *vstop = 1;
    raise_flag(err, MKG_DEV_TIMEOUT);
    return false;
  };
  if (threadIdx.x == 0) {
    for (int k = 0; k < kColsumStages; ++k) {
      mbar_init(&full[k], 1);
      mbar_init(&empty[k], 1);
    }
    mbar_init_fence();
    stop = 0;
    issued = 0;
    consumed = 0;
  }
  __syncthreads();
  float s = 0.0f;
  if (warp == 1) {  // producer
    if (lane == 0) {
      int64_t t = 0;
      for (; t < ntiles && !*vstop; ++t) {
        const int slot = (int)(t % kColsumStages);
        const int64_t round = t / kColsumStages;
        if (round > 0) {
          if (!wait(&empty[slot], (uint32_t)((round - 1) & 1))) break;
          fence_proxy_async_smem();
        }
        mbar_expect_tx(&full[slot], kTileBytes);
        tma_load_2d(&buf[slot][0][0], &ymap, (int32_t)c0, (int32_t)(t * kColsumRows), &full[slot]);
      }
      issued = t;
    }
  } else {  // consumer
    int64_t t = 0;
    for (; t < ntiles; ++t) {
      const int slot = (int)(t % kColsumStages);
      const int64_t round = t / kColsumStages;
      const bool ok = wait(&full[slot], (uint32_t)(round & 1));  // every lane observes the phase
      if (!__all_sync(0xffffffffu, ok)) break;
      const int64_t left = q.E - t * kColsumRows;
      const int rows = left < kColsumRows ? (int)left : kColsumRows;
      int r = 0;
      for (; r + 8 <= rows; r += 8) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = buf[slot][r + k][lane];
#pragma unroll
        for (int k = 0; k < 8; ++k) s = __fadd_rn(s, v[k]);
      }
      for (; r < rows; ++r) s = __fadd_rn(s, buf[slot][r][lane]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (lane == 0) consumed = t;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // a copy that was issued but whose tile was never consumed must land before the block
    // exits (its shared memory is released then); each wait is bounded
    for (long long t = consumed; t < issued; ++t) {
      const int slot = (int)(t % kColsumStages);
      if (!mbar_wait_bounded(&full[slot], (uint32_t)((t / kColsumStages) & 1), kWaitPolls)) {
        raise_flag(err, MKG_DEV_TIMEOUT);
        break;
      }
    }
  }
  if (warp == 0 && lane < ncols) d[c0 + lane] = fmaxf(s, 1e-7f);
}

// Tensor map of a row-major [rows][cols] fp32 matrix with a 64 x 32 box (cols is a multiple
// of 4, so every row stride and box start is 16-byte aligned).
int make_rows_map(CUtensorMap* map, const float* base, int64_t rows, int64_t cols) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr) != cudaSuccess ||
        qr != cudaDriverEntryPointSuccess)
      fn = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }();
  if (encode == nullptr) { set_error("cuTensorMapEncodeTiled is unavailable"); return MKG_ERR_CUDA; }
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
  const cuuint32_t box[2] = {32, kColsumRows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) { set_error("cuTensorMapEncodeTiled failed (%d)", (int)r); return MKG_ERR_CUDA; }
  return MKG_OK;
}

__global__ void normalize_plain_kernel(const float* __restrict__ y, const float* __restrict__ d, ProofDims q,
                                       float* __restrict__ x, uint8_t* __restrict__ act,
                                       const int32_t* __restrict__ push_ptr, const int32_t* __restrict__ capdeg,
                                       int64_t* __restrict__ msgs) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  long long local_msgs = 0;
  for (int64_t task = warp0; task < q.E * q.nch; task += nwarps) {
    const int64_t row = task / q.nch, chunk = task % q.nch;
    const int64_t col = chunk * kChunk + 4 * lane;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    if (col < q.BLP) {
      const float4 v = *reinterpret_cast<const float4*>(y + row * q.BLP + col);
      const float4 dd = *reinterpret_cast<const float4*>(d + col);
      o.x = v.x != 0.f ? __fdiv_rn(v.x, dd.x) : 0.f;
      o.y = v.y != 0.f ? __fdiv_rn(v.y, dd.y) : 0.f;
      o.z = v.z != 0.f ? __fdiv_rn(v.z, dd.z) : 0.f;
      o.w = v.w != 0.f ? __fdiv_rn(v.w, dd.w) : 0.f;
      *reinterpret_cast<float4*>(x + row * q.BLP + col) = o;
    }
    const int nz = f4_count(o);
    const unsigned any = __ballot_sync(0xffffffffu, nz > 0);
    int tot = nz;
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, s);
    if (lane == 0) {
      act[row * q.nch + chunk] = any ? 1 : 0;
      if (tot) local_msgs += (long long)tot * (capdeg ? capdeg[row] : push_ptr[row + 1] - push_ptr[row]);
    }
  }
  if (lane == 0 && local_msgs) atomicAdd(reinterpret_cast<unsigned long long*>(msgs), (unsigned long long)local_msgs);
}

// out[b][e] = reduce_l X[e][b*L + l] (sum: sum_sp_3d; max: max over rules of the
// normalised state, norm_sp_3d_max).  A 32-entity x 32-query tile goes through shared
// memory so that both the reads and the [B][E] writes are coalesced.  For the max the
// value is divided by d first (norm_sp_3d), the division is fused here.
template <bool MAX>
__global__ void rows_to_queries_kernel(const float* __restrict__ x, const float* __restrict__ d, ProofDims q,
                                       float* __restrict__ out) {
  __shared__ float tile[32][33];
  const int64_t e0 = blockIdx.x * 32, b0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int r = ty; r < 32; r += 8) {
    const int64_t e = e0 + r, b = b0 + tx;
    float v = 0.0f;
    if (e < q.E && b < q.B) {
      const float* src = x + e * q.BLP + b * q.L;
      if (MAX) {
        v = 0.0f;
        for (int64_t l = 0; l < q.L; ++l) {
          float t = src[l];
          if (t != 0.0f) t = __fdiv_rn(t, d[b * q.L + l]);
          v = fmaxf(v, t);
        }
      } else {
        for (int64_t l = 0; l < q.L; ++l) v = __fadd_rn(v, src[l]);
      }
    }
    tile[r][tx] = v;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int64_t b = b0 + r, e = e0 + tx;
    if (b < q.B && e < q.E) out[b * q.E + e] = tile[tx][r];
  }
}

// ------------------------------------------------------------------ backward
// Seed: dX_K[e][c] = G[b][e] where X_K[e][c] != 0 (the reference's sparse result carries
// gradient only on its keys), and S[c] = sum_e dX_K[e][c] * Y_{K-1}[e][c].
constexpr int kSeedTiles = 4;   // 32-entity tiles per block of seed_grad_kernel
constexpr int kSeedRows = 4;    // rows whose loads a thread issues together

// Block = 32 queries (the contiguous columns [32 L by, 32 L (by + 1)) of every row, 16-byte
// aligned since BLP is a multiple of 4) x kSeedTiles tiles of 32 entities.  The G tile goes
// through shared memory; X_K, Y_{K-1} and dX_K are streamed in float4s.  A thread keeps one
// float4 column of the segment for the whole block (rows step by 256 / float4s per row), so the
// queries of its 4 columns are found once and its S partials stay in registers; they are summed
// in shared memory at the end.  Segments wider than 256 float4s (L > 32) take several column
// passes and add S with global atomics.  A float4 that reaches past B L covers padding columns,
// which hold zeros in X_K and get zeros in dX_K.
__global__ void __launch_bounds__(256, 4) seed_grad_kernel(const float* __restrict__ g, const float* __restrict__ xk,
                                                       const float* __restrict__ ylast, ProofDims q,
                                                       float* __restrict__ dx, double* __restrict__ s) {
  __shared__ float tile[32][33];  // [query][entity] of G
  __shared__ double part[1024];   // S of the block's columns (width <= 1024 on the register path)
  const int tid = threadIdx.x;
  const int64_t b0 = blockIdx.y * 32;
  const int nb = static_cast<int>(q.B - b0 < 32 ? q.B - b0 : 32);
  const int L = static_cast<int>(q.L);
  const int64_t c0 = b0 * L;
  const int width = nb * L;         // columns of the block's queries
  const int nf4 = (width + 3) / 4;  // float4s per row (the last may reach into padding)
  const bool fixed = nf4 <= 256;    // one column pass: S partials in registers
  const int cols = fixed ? nf4 : 256;
  const int rpp = 256 / cols;       // rows per pass
  const int cf = tid % cols, rr = tid / cols;
  const bool worker = rr < rpp;
  for (int i = tid; i < 1024; i += 256) part[i] = 0.0;
  float sacc[4] = {0.f, 0.f, 0.f, 0.f};  // over at most 128 rows; fp64 from the block sums on
  for (int t = 0; t < kSeedTiles; ++t) {
    const int64_t e0 = ((int64_t)blockIdx.x * kSeedTiles + t) * 32;
    if (e0 >= q.E) break;
    const int rows = static_cast<int>(q.E - e0 < 32 ? q.E - e0 : 32);
    __syncthreads();  // the previous tile is consumed (and part is zeroed)
    for (int i = tid; i < 32 * 32; i += 256) {
      const int b = i >> 5, e = i & 31;
      tile[b][e] = (b < nb && e < rows) ? g[(b0 + b) * q.E + e0 + e] : 0.0f;
    }
    __syncthreads();
    if (!worker) continue;
    for (int f = cf; f < nf4; f += cols) {
      const int j0 = 4 * f;
      int bq[4];
      bool ok[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        ok[k] = j0 + k < width;
        bq[k] = ok[k] ? (j0 + k) / L : 0;
      }
      for (int r0 = rr; r0 < rows; r0 += rpp * kSeedRows) {
        float4 xv[kSeedRows], yv[kSeedRows];
#pragma unroll
        for (int u = 0; u < kSeedRows; ++u) {
          const int r = r0 + u * rpp;
          if (r < rows) {
            const int64_t off = (e0 + r) * q.BLP + c0 + j0;
            xv[u] = *reinterpret_cast<const float4*>(xk + off);
            yv[u] = *reinterpret_cast<const float4*>(ylast + off);
          }
        }
#pragma unroll
        for (int u = 0; u < kSeedRows; ++u) {
          const int r = r0 + u * rpp;
          if (r >= rows) break;
          const float xs[4] = {xv[u].x, xv[u].y, xv[u].z, xv[u].w};
          const float ys[4] = {yv[u].x, yv[u].y, yv[u].z, yv[u].w};
          float o[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float dv = (ok[k] && xs[k] != 0.0f) ? tile[bq[k]][r] : 0.0f;
            o[k] = dv;
            if (fixed) sacc[k] = fmaf(dv, ys[k], sacc[k]);
            else if (dv != 0.0f) atomicAdd(s + c0 + j0 + k, (double)(dv * ys[k]));
          }
          *reinterpret_cast<float4*>(dx + (e0 + r) * q.BLP + c0 + j0) = make_float4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
  if (fixed) {
    if (worker) {
      const int j0 = 4 * cf;
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (j0 + k < width && sacc[k] != 0.0f) atomicAdd(part + j0 + k, (double)sacc[k]);
    }
    __syncthreads();
    for (int j = tid; j < width; j += 256)
      if (part[j] != 0.0) atomicAdd(s + c0 + j, part[j]);
  }
}

// Gradient of x = (y / d) * min(d, 1) with d = column sum of y (only y != 0 entries):
// dy = dx * (c / d) + S * coef, coef = -1 / d^2 when d > 1 and 0 when d <= 1 (where
// min(d, 1) = d and the two terms cancel).  A warp takes kNbTasks (row, 128-column chunk)
// tasks at a time and skips the chunks where Y_h is zero (yact): dY is zero there, and the
// backward pull reads dY only in chunks whose yact is set, so those chunks are not written.
// The same launch zeroes the rows of dx_next (the slab this hop's pull writes) that several push
// tasks add into: this kernel does not read that slab, the previous hop's did.
constexpr int kNbTasks = 4;

__global__ void __launch_bounds__(256, 4) normalize_mass_backward_kernel(
    const float* __restrict__ dx, const float* __restrict__ y, const float* __restrict__ dsum,
    const double* __restrict__ s, const uint8_t* __restrict__ yact, ProofDims q, float* __restrict__ dy,
    const int4* __restrict__ push_tasks, int64_t num_push_tasks, float* __restrict__ dx_next) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t total = q.E * q.nch;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t t = warp0; t < num_push_tasks; t += nwarps) {
    const int4 tk = push_tasks[t];
    if ((tk.w & (kTaskFirst | kTaskPartial)) != (kTaskFirst | kTaskPartial)) continue;
    float4* row = reinterpret_cast<float4*>(dx_next + (int64_t)tk.x * q.BLP);
    for (int64_t j = lane; j < q.BLP / 4; j += 32) row[j] = zero;
  }
  for (int64_t t0 = warp0 * kNbTasks; t0 < total; t0 += nwarps * kNbTasks) {
    const int64_t row0 = t0 / q.nch, chunk0 = t0 % q.nch;
    bool on[kNbTasks];
    float4 g[kNbTasks], v[kNbTasks];
    {
      int64_t row = row0, chunk = chunk0;
#pragma unroll
      for (int u = 0; u < kNbTasks; ++u) {
        const int64_t col = chunk * kChunk + 4 * lane;
        on[u] = t0 + u < total && col < q.BLP && yact[t0 + u] != 0;
        g[u] = on[u] ? *reinterpret_cast<const float4*>(dx + row * q.BLP + col) : zero;
        v[u] = on[u] ? *reinterpret_cast<const float4*>(y + row * q.BLP + col) : zero;
        if (++chunk == q.nch) { chunk = 0; ++row; }
      }
    }
    int64_t row = row0, chunk = chunk0;
#pragma unroll
    for (int u = 0; u < kNbTasks; ++u) {
      const int64_t col = chunk * kChunk + 4 * lane;
      if (on[u]) {
        const float4 d = *reinterpret_cast<const float4*>(dsum + col);
        // S rounded to fp32 once, from its fp64 sum
        const double2 s01 = *reinterpret_cast<const double2*>(s + col);
        const double2 s23 = *reinterpret_cast<const double2*>(s + col + 2);
        float gi[4] = {g[u].x, g[u].y, g[u].z, g[u].w}, vi[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        float di[4] = {d.x, d.y, d.z, d.w}, o[4];
        const float si[4] = {(float)s01.x, (float)s01.y, (float)s23.x, (float)s23.y};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float r = 0.0f;
          if (vi[k] != 0.0f) {
            const float dd = di[k];
            const float c = fminf(dd, 1.0f);
            const float coef = dd <= 1.0f ? 0.0f : -__fdiv_rn(1.0f, dd * dd);
            r = gi[k] * __fdiv_rn(c, dd) + si[k] * coef;
          }
          o[k] = r;
        }
        *reinterpret_cast<float4*>(dy + row * q.BLP + col) = make_float4(o[0], o[1], o[2], o[3]);
      }
      if (++chunk == q.nch) { chunk = 0; ++row; }
    }
  }
}

__device__ __forceinline__ float edge_grad_scale(const EdgeFactor& f, int64_t fact) {
  if (f.weight == nullptr) return 0.0f;
  const float ew = f.weight[fact];
  if (f.is_score) return 1.0f / fmaxf(ew, 1e-12f);
  const float z = -ew * f.scale;
  const float sg = static_cast<float>(1.0 / (1.0 + exp(static_cast<double>(z))));
  return f.scale * (1.0f - sg);
}

// Reduce-scatter of 4 per-lane partial sums: afterwards lane l holds, for edge
// ((l >> 3) & 3), the sum of that edge's partials over all 32 lanes (6 shuffles).
__device__ __forceinline__ float reduce_scatter4(const float (&v)[4]) {
  const int lane = threadIdx.x & 31;
  const bool h4 = lane & 16, h3 = lane & 8;
  float a[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float send = h4 ? v[k] : v[k + 2];
    const float keep = h4 ? v[k + 2] : v[k];
    a[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  float c = (h3 ? a[1] : a[0]) + __shfl_xor_sync(0xffffffffu, h3 ? a[0] : a[1], 8);
  c += __shfl_xor_sync(0xffffffffu, c, 4);
  c += __shfl_xor_sync(0xffffffffu, c, 2);
  c += __shfl_xor_sync(0xffffffffu, c, 1);
  return c;
}

// Transposed hop over the push list (row = sending entity s, records = its messages):
//   dX[s][c]   = [X[s][c] != 0] (dY[s][c] w[n-1][c] + sum_ch w[ch][c] sum_{e in ch} dY[d_e][c] m_e)
//   dW[ch][c] += X[s][c] sum_{e in ch} dY[d_e][c] m_e     (shared-memory partial per block)
//   dEdge[f]  += (sum_c dY[d][c] X[s][c] w[ch][c]) m g(f)
//   S_prev[c] += dX[s][c] Y_prev[s][c]                   (for the next lower hop)
// Records of a push row come grouped by channel, so dY * m is summed per channel run and
// folded into dX and dW once per run, and the edge-score gradient uses the run's X * W[ch]
// (one rule-weight load per run).  Only records whose destination row holds a non-zero Y_h
// value in this chunk are visited (dY_h is zero elsewhere).  Rule weights are read from
// global memory (L1-resident chunk) so that only dW occupies shared memory: 4 blocks per SM
// (64 registers, a few bytes spilled; the capped loop, which spills more there, keeps 3).
// Acc: the shared-memory accumulator of the rule-weight gradient, double where [n, 128] of it
// fits (each fp64 product added once: the fp32 partials of many terms of both signs drifted past
// 1e-5 of the result), float for wider channel counts.
template <bool CAP, typename Acc>
__global__ void __launch_bounds__(kBwdWarps * 32, CAP ? 3 : 4) bwd_pull_kernel(
    const int4* __restrict__ tasks, int64_t ntasks, const mkg_adj_edge* __restrict__ edges, ProofDims q,
    const float* __restrict__ wt, const float* __restrict__ x, const uint8_t* __restrict__ act,
    const uint8_t* __restrict__ yact, const float* __restrict__ dy, const float* __restrict__ yprev,
    float* __restrict__ dx, double* __restrict__ dwt, double* __restrict__ sprev, float* __restrict__ grad_edge,
    int64_t num_facts, EdgeFactor ef, int32_t* __restrict__ queue, const int2* __restrict__ rcap,
    const uint8_t* __restrict__ take, unsigned* err) {
  extern __shared__ double smem[];
  Acc* dws = reinterpret_cast<Acc*>(smem);  // [n][128] rule-weight gradient (conflict-free: [ch][k][lane])
  // [4][32] S_prev partials in fp64 (dX Y terms of both signs cancel in S)
  double* cs = reinterpret_cast<double*>(dws + q.n * kChunk);
  const int lane = threadIdx.x & 31;
  const int64_t chunk = blockIdx.y;
  const int64_t col0 = chunk * kChunk;
  const int64_t col = col0 + 4 * lane;
  const bool colok = col < q.BLP;
  for (int64_t i = threadIdx.x; i < q.n * kChunk; i += blockDim.x) dws[i] = Acc(0);
  for (int i = threadIdx.x; i < kChunk; i += blockDim.x) cs[i] = 0.0;
  __syncthreads();
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  // rule weights of this chunk from global memory (L1-resident): W[ch] at wt + ch * BLP + col
  auto wload = [&](int64_t ch) -> float4 {
    return colok ? __ldg(reinterpret_cast<const float4*>(wt + ch * q.BLP + col)) : make_float4(0.f, 0.f, 0.f, 0.f);
  };
  TaskCursor cursor(queue + chunk * kQueueStride, ntasks);
  int64_t t;
  while (cursor.next(t)) {
    const int4 tk = tasks[t];
    const int64_t row = tk.x;
    const bool active = act[row * q.nch + chunk] != 0;
    float4 gx = zero;
    if (active) {
      const float4 xr = colok ? *reinterpret_cast<const float4*>(x + row * q.BLP + col) : zero;
      if ((tk.w & kTaskFirst) && colok && yact[row * q.nch + chunk] != 0) {  // dY_h[row] is zero elsewhere
        const float4 ds = *reinterpret_cast<const float4*>(dy + row * q.BLP + col);
        const float4 wi = wload(q.n - 1);
        gx = f4_mul(ds, wi);
        Acc* dwi = dws + (q.n - 1) * kChunk;
        if (ds.x != 0.f) atomicAdd(dwi + 0 * 32 + lane, Acc(ds.x) * Acc(xr.x));
        if (ds.y != 0.f) atomicAdd(dwi + 1 * 32 + lane, Acc(ds.y) * Acc(xr.y));
        if (ds.z != 0.f) atomicAdd(dwi + 2 * 32 + lane, Acc(ds.z) * Acc(xr.z));
        if (ds.w != 0.f) atomicAdd(dwi + 3 * 32 + lane, Acc(ds.w) * Acc(xr.w));
      }
      float4 run = zero;  // sum of dY * m over the current channel run
      int cur = -1;
      float4 wcur = zero;  // W[cur] of this chunk, loaded once per run
      float4 xw = zero;    // X[s] * W[cur]: the run's factor of the edge-score gradient
      auto flush = [&]() {
        if (cur < 0) return;
        const float4 wc = wcur;
        gx.x = fmaf(run.x, wc.x, gx.x); gx.y = fmaf(run.y, wc.y, gx.y);
        gx.z = fmaf(run.z, wc.z, gx.z); gx.w = fmaf(run.w, wc.w, gx.w);
        Acc* dwc = dws + cur * kChunk;
        if (run.x != 0.f) atomicAdd(dwc + 0 * 32 + lane, Acc(run.x) * Acc(xr.x));
        if (run.y != 0.f) atomicAdd(dwc + 1 * 32 + lane, Acc(run.y) * Acc(xr.y));
        if (run.z != 0.f) atomicAdd(dwc + 2 * 32 + lane, Acc(run.z) * Acc(xr.z));
        if (run.w != 0.f) atomicAdd(dwc + 3 * 32 + lane, Acc(run.w) * Acc(xr.w));
        run = zero;
      };
      for (int base = tk.y; base < tk.z; base += 32) {
        const int cnt = min(32, tk.z - base);
        int4 rec = make_int4(0, 0, 0, 0);
        int2 rc = make_int2(-1, 0);
        bool live = false;
        if (lane < cnt) {
          rec = reinterpret_cast<const int4*>(edges)[base + lane];
          if (CAP) rc = rcap[base + lane];
          if (rec.x < 0 || rec.x >= q.E || rec.y < 0 || rec.y >= q.n - 1) raise_flag(err, MKG_DEV_BAD_COL);
          else if (CAP && rc.x >= q.ngroups) raise_flag(err, MKG_DEV_BAD_ENTRY);
          else live = yact[(int64_t)rec.x * q.nch + chunk] != 0;  // dY is zero where Y is
        }
        unsigned pending = __ballot_sync(0xffffffffu, live);
        while (pending) {
          int nb[kBatch], ch[kBatch], fa[kBatch];
          float m[kBatch];
          bool ok[kBatch];
          int src[kBatch];  // lane that loaded the record
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            ok[u] = pending != 0;
            const int jj = ok[u] ? __ffs(pending) - 1 : 0;
            pending &= pending - 1;
            nb[u] = __shfl_sync(0xffffffffu, rec.x, jj);
            ch[u] = __shfl_sync(0xffffffffu, rec.y, jj);
            fa[u] = __shfl_sync(0xffffffffu, rec.z, jj);
            m[u] = __int_as_float(__shfl_sync(0xffffffffu, rec.w, jj));
            src[u] = jj;
          }
          float4 gv[kBatch];
#pragma unroll
          for (int u = 0; u < kBatch; ++u)
            gv[u] = (ok[u] && colok) ? *reinterpret_cast<const float4*>(dy + (int64_t)nb[u] * q.BLP + col) : zero;
          if (CAP) {
            unsigned tw[kBatch];
            int tp[kBatch];
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
              const int2 cr = make_int2(__shfl_sync(0xffffffffu, rc.x, src[u]), __shfl_sync(0xffffffffu, rc.y, src[u]));
              tw[u] = (ok[u] && colok && cr.x >= 0)
                          ? __ldg(reinterpret_cast<const unsigned*>(take + (int64_t)cr.x * q.tblp +
                                                                    take_lane_offset(chunk, lane)))
                          : 0xFFFFFFFFu;
              tp[u] = cr.x >= 0 ? cr.y : -1;  // -1: a record of an uncapped row
            }
#pragma unroll
            for (int u = 0; u < kBatch; ++u)
              if (tp[u] >= 0) gv[u] = cap_masked(gv[u], tw[u], tp[u]);  // uniform over the warp
          }
          float ep[kBatch];
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            ep[u] = 0.0f;
            if (!ok[u]) continue;
            if (ch[u] != cur) {
              flush();
              cur = ch[u];
              wcur = wload(cur);
              xw = f4_mul(xr, wcur);
            }
            run.x = fmaf(gv[u].x, m[u], run.x); run.y = fmaf(gv[u].y, m[u], run.y);
            run.z = fmaf(gv[u].z, m[u], run.z); run.w = fmaf(gv[u].w, m[u], run.w);
            if (grad_edge != nullptr) {
              ep[u] = gv[u].x * xw.x + gv[u].y * xw.y + gv[u].z * xw.z + gv[u].w * xw.w;
            }
          }
          if (grad_edge != nullptr) {
            const float tot = reduce_scatter4(ep);
            const int idx = (lane >> 3) & 3;
            int f = -1;
            float mm = 0.0f;
#pragma unroll
            for (int u = 0; u < kBatch; ++u)
              if (idx == u && ok[u]) { f = fa[u]; mm = m[u]; }
            if ((lane & 7) == 0 && f >= 0 && tot != 0.0f) {
              if (f < num_facts) atomicAdd(grad_edge + f, tot * mm * edge_grad_scale(ef, f));
              else raise_flag(err, MKG_DEV_BAD_FACT);
            }
          }
        }
      }
      flush();
      // only present entries of X carry a gradient
      gx.x = xr.x != 0.f ? gx.x : 0.f; gx.y = xr.y != 0.f ? gx.y : 0.f;
      gx.z = xr.z != 0.f ? gx.z : 0.f; gx.w = xr.w != 0.f ? gx.w : 0.f;
    }
    if (colok) {
      float* dr = dx + row * q.BLP + col;
      if (tk.w & kTaskPartial) {
        if (active) { atomicAdd(dr + 0, gx.x); atomicAdd(dr + 1, gx.y); atomicAdd(dr + 2, gx.z); atomicAdd(dr + 3, gx.w); }
      } else {
        *reinterpret_cast<float4*>(dr) = gx;
      }
      if (sprev != nullptr && active) {  // each product added once, in fp64
        const float4 yp = *reinterpret_cast<const float4*>(yprev + row * q.BLP + col);
        if (yp.x != 0.f) atomicAdd(cs + 0 * 32 + lane, (double)(gx.x * yp.x));
        if (yp.y != 0.f) atomicAdd(cs + 1 * 32 + lane, (double)(gx.y * yp.y));
        if (yp.z != 0.f) atomicAdd(cs + 2 * 32 + lane, (double)(gx.z * yp.z));
        if (yp.w != 0.f) atomicAdd(cs + 3 * 32 + lane, (double)(gx.w * yp.w));
      }
    }
  }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < q.n * kChunk; i += blockDim.x) {
    const int64_t ch = i / kChunk, r = i % kChunk, l = r % 32, k = r / 32;
    const int64_t c = col0 + 4 * l + k;
    if (c < q.BLP && dws[i] != Acc(0)) atomicAdd(dwt + ch * q.BLP + c, static_cast<double>(dws[i]));
  }
  if (sprev != nullptr) {
    for (int i = threadIdx.x; i < kChunk; i += blockDim.x) {
      const int l = i % 32, k = i / 32;
      const int64_t c = col0 + 4 * l + k;
      if (c < q.BLP && cs[i] != 0.0) atomicAdd(sprev + c, cs[i]);
    }
  }
}

// ------------------------------------------------------------------ decode top-k
// One block per query row: candidate keys (bounded score << 32 | ~tail), MSB radix select
// of the k-th largest, then a bitonic sort of the selected keys in shared memory.
constexpr int kTopkThreads = 1024;
constexpr int kTopkMax = 1024;

__device__ __forceinline__ unsigned long long candidate_key(float raw, int64_t e) {
  if (!(raw != 0.0f)) return 0ull;
  const float xv = fmaxf(raw, 0.0f);
  const float ex = static_cast<float>(exp(-static_cast<double>(xv)));
  const float score = 1.0f - ex;  // bound_sparse_scores, float32 arithmetic
  return (static_cast<unsigned long long>(__float_as_uint(score)) << 32) |
         static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(e));
}

// every stored entry is a candidate (a sparse state's explicit zeros get score 0)
__device__ __forceinline__ unsigned long long stored_candidate_key(float raw, int64_t e) {
  const float xv = fmaxf(raw, 0.0f);
  const float ex = static_cast<float>(exp(-static_cast<double>(xv)));
  const float score = 1.0f - ex;
  return (static_cast<unsigned long long>(__float_as_uint(score)) << 32) |
         static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(e));
}

// Row sources of the decode top-k: a dense [B, E] raw-score array (zeros are absent entries),
// or a key-sorted sparse state (keys b * E + e ascending; every stored entry is a candidate).
struct DenseTopkRows {
  const float* raw;
  int64_t E;
  __device__ void range(int64_t b, int64_t& lo, int64_t& hi) const { lo = b * E; hi = lo + E; }
  __device__ unsigned long long key(int64_t i, int64_t lo) const { return candidate_key(raw[i], i - lo); }
};

// candidate keys of a sparse state, formed once (the radix passes read them again and again)
__global__ void sparse_candidate_keys_kernel(const int64_t* __restrict__ keys, const float* __restrict__ vals,
                                             int64_t nnz, int64_t E, unsigned long long* __restrict__ cand) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nnz; i += (int64_t)gridDim.x * blockDim.x)
    cand[i] = stored_candidate_key(vals[i], keys[i] % E);
}

struct SparseTopkRows {
  const int64_t* keys;
  const unsigned long long* cand;
  int64_t nnz, E;
  __device__ int64_t lower_bound(int64_t v) const {
    int64_t lo = 0, hi = nnz;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (keys[mid] < v) lo = mid + 1; else hi = mid;
    }
    return lo;
  }
  __device__ void range(int64_t b, int64_t& lo, int64_t& hi) const {
    lo = lower_bound(b * E);
    hi = lower_bound((b + 1) * E);
  }
  __device__ unsigned long long key(int64_t i, int64_t) const { return cand[i]; }
};

template <class Rows>
__global__ void __launch_bounds__(kTopkThreads) topk_rows_kernel(Rows rows, int64_t k, int64_t* __restrict__ tails,
                                                                 float* __restrict__ scores,
                                                                 int64_t* __restrict__ counts) {
  typedef cub::BlockReduce<long long, kTopkThreads> CandReduce;
  __shared__ typename CandReduce::TempStorage reduce_tmp;
  __shared__ unsigned int hist[256];
  __shared__ unsigned long long sel[kTopkMax];
  __shared__ unsigned long long prefix_s;
  __shared__ long long need_s;
  __shared__ int nsel;
  __shared__ long long ncand_s;
  const int64_t b = blockIdx.x;
  int64_t lo, hi;
  rows.range(b, lo, hi);
  if (threadIdx.x == 0) { ncand_s = 0; nsel = 0; prefix_s = 0ull; }
  __syncthreads();
  long long my = 0;
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) my += rows.key(i, lo) != 0ull;
  my = CandReduce(reduce_tmp).Sum(my);
  if (threadIdx.x == 0) { ncand_s = my; need_s = my < k ? my : k; }
  __syncthreads();
  const long long ncand = ncand_s;
  const long long kk = need_s;
  unsigned long long thresh = 1ull;  // every candidate key is > 0
  if (ncand > k) {
    // MSB radix select: the kk-th largest key among the candidates
    unsigned long long prefix = 0ull, mask = 0ull;
    long long need = kk;
    for (int shift = 56; shift >= 0; shift -= 8) {
      for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
      __syncthreads();
      for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const unsigned long long key = rows.key(i, lo);
        if (key != 0ull && (key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xffu], 1u);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        long long acc = 0;
        int dsel = 0;
        for (int dgt = 255; dgt >= 0; --dgt) {
          if (acc + hist[dgt] >= need) { dsel = dgt; break; }
          acc += hist[dgt];
        }
        need_s = need - acc;
        prefix_s = prefix | (static_cast<unsigned long long>(dsel) << shift);
      }
      __syncthreads();
      need = need_s;
      prefix = prefix_s;
      mask |= 0xffull << shift;
      __syncthreads();
    }
    thresh = prefix;  // keys are unique (distinct tails): exactly kk keys are >= thresh
  }
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const unsigned long long key = rows.key(i, lo);
    if (key != 0ull && key >= thresh) {
      int pos = atomicAdd(&nsel, 1);
      if (pos < kTopkMax) sel[pos] = key;
    }
  }
  __syncthreads();
  const int m = min(nsel, kTopkMax);
  int p2 = 1;
  while (p2 < m) p2 <<= 1;
  for (int i = threadIdx.x; i < p2; i += blockDim.x)
    if (i >= m) sel[i] = 0ull;
  __syncthreads();
  // bitonic sort, descending
  for (int size = 2; size <= p2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < p2; i += blockDim.x) {
        int j = i ^ stride;
        if (j > i) {
          bool desc = (i & size) == 0;
          unsigned long long a = sel[i], c = sel[j];
          if (desc ? (a < c) : (a > c)) { sel[i] = c; sel[j] = a; }
        }
      }
      __syncthreads();
    }
  }
  for (int64_t j = threadIdx.x; j < k; j += blockDim.x) {
    if (j < m) {
      unsigned long long key = sel[j];
      tails[b * k + j] = static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull));
      scores[b * k + j] = __uint_as_float(static_cast<uint32_t>(key >> 32));
    } else {
      tails[b * k + j] = -1;
      scores[b * k + j] = 0.0f;
    }
  }
  if (threadIdx.x == 0) counts[b] = m;
}

constexpr size_t kBwdSmemMax = 200 * 1024;
// shared memory of the backward pull with fp64 (f64) or fp32 rule-weight partials
size_t bwd_smem(const ProofDims& q, bool f64 = false) {
  return (f64 ? 8 : 4) * (size_t)q.n * kChunk + 8 * (size_t)kChunk;
}

// Columns per lane of the forward pull: 8 (two float4) for batches wider than 128
// columns; MKG_FWD_VEC=1|2 overrides (a tuning knob).
int fwd_vec_knob(const ProofDims& q) {
  static int forced = [] {
    const char* v = getenv("MKG_FWD_VEC");
    return v ? atoi(v) : 0;
  }();
  if (forced == 1 || forced == 2) return forced;
  return q.BLP > kChunk ? 2 : 1;
}

int check_proof(const mkg_graph* g, const mkg_adjacency* adj, const mkg_proof_params* p) {
  MKG_REQUIRE(g && adj && p, "proof: null argument");
  MKG_REQUIRE(p->B >= 1 && p->L >= 1 && p->hops >= 1 && p->R >= 1, "proof: B, L, R, hops must be positive");
  MKG_REQUIRE(p->E == g->num_entities, "proof: E does not match the graph");
  MKG_REQUIRE(adj->pull_tasks && adj->push_tasks && adj->num_pull_tasks > 0 && adj->num_push_tasks > 0 &&
                  adj->pull && adj->push && adj->pull_ptr && adj->push_ptr,
              "proof: adjacency has no task lists (call mkg_adjacency_build and read the task counts)");
  if (p->topk_edges < (int64_t(1) << 60)) {
    const mkg_cap_index* ix = p->cap_index;
    if (p->topk_edges < 0 || p->topk_edges > MKG_DENSE_CAP_MAX) {
      set_error("proof: the fused loop takes edge caps in [0, %d] (got %lld); larger caps go through "
                "mkg_hop_forward", MKG_DENSE_CAP_MAX, (long long)p->topk_edges);
      return MKG_ERR_UNSUPPORTED;
    }
    MKG_REQUIRE(ix != nullptr, "proof: a capped loop needs the cap index (mkg_cap_index_build)");
    MKG_REQUIRE(ix->cap == p->topk_edges, "proof: the cap index was built for cap %lld, not %lld",
                (long long)ix->cap, (long long)p->topk_edges);
    MKG_REQUIRE(ix->pull_cap && ix->push_cap && ix->capped_degree && ix->num_slots >= 0 && ix->num_groups >= 0 &&
                    (ix->num_slots == 0 || (ix->slot_entity && ix->slot_dir && ix->slot_group)),
                "proof: incomplete cap index");
  }
  ProofDims q = proof_dims(*p);
  MKG_REQUIRE(bwd_smem(q) <= kBwdSmemMax, "proof: too many relation channels (%lld) for the shared-memory "
              "staging of the rule weights", (long long)q.n);
  return MKG_OK;
}

}  // namespace

size_t proof_workspace_bytes(const mkg_proof_params* p) {
  return proof_layout(proof_dims(*p)).total + 256;
}

static int set_smem(const void* fn, size_t bytes) {
  MKG_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return MKG_OK;
}

// Forward of the hop loop (sum) or of the max loop; keeps every hop in the workspace.
static int run_forward(const mkg_graph* g, const mkg_adjacency* adj, const int64_t* heads, const float* w_hops,
                       const mkg_proof_params* p, bool max_mode, void* ws, size_t ws_bytes, float* out,
                       int64_t* messages_out, unsigned* err, cudaStream_t st) {
  int rc = check_proof(g, adj, p);
  if (rc) return rc;
  MKG_REQUIRE(heads && w_hops && out, "proof: null input / output");
  const ProofDims q = proof_dims(*p);
  Slab S{static_cast<char*>(ws), proof_layout(q), q};
  MKG_REQUIRE(ws && ws_bytes >= S.lay.total, "proof: workspace too small (%zu < %zu)", ws_bytes, S.lay.total);
  const size_t slab = 4 * (size_t)q.E * q.BLP;
  const int pb = persistent_blocks(4);
  transpose_w_kernel<<<grid_for(q.hops * q.n * q.BLP, 256, pb), 256, 0, st>>>(w_hops, q, S.wt(0));
  MKG_LAUNCHED("transpose_w_kernel");
  forward_setup_kernel<<<pb, 256, 0, st>>>(
      heads, reinterpret_cast<const int4*>(adj->pull_tasks), adj->num_pull_tasks, q, S.act(0),
      (int64_t)(S.lay.yact - S.lay.act) + q.hops * q.E * q.nch, S.y(0), (int64_t)(a256(slab) / 4), S.x(0), S.d(0),
      S.queue(), q.hops * q.nch * kQueueStride, S.msgs());
  MKG_LAUNCHED("forward_setup_kernel");
  const mkg_cap_index* ix = q.cap >= 0 ? p->cap_index : nullptr;
  const int32_t* capdeg = ix ? ix->capped_degree : nullptr;
  const int2* pull_cap = ix ? reinterpret_cast<const int2*>(ix->pull_cap) : nullptr;
  init_state_kernel<<<grid_for(q.BL, 256, pb), 256, 0, st>>>(heads, q, S.x(0), S.act(0), adj->push_ptr, capdeg,
                                                             S.msgs(), err);
  MKG_LAUNCHED("init_state_kernel");
  // 256-column chunks (8 columns per lane) when the batch is wide enough
  const int vec = fwd_vec_knob(q);
  const int64_t nfch = (q.BLP + 128 * vec - 1) / (128 * vec);
  const void* fwd_fn = max_mode ? (vec == 2 ? (const void*)fwd_pull_kernel<true, 2, false> : (const void*)fwd_pull_kernel<true, 1, false>)
                                : (vec == 2 ? (const void*)fwd_pull_kernel<false, 2, false> : (const void*)fwd_pull_kernel<false, 1, false>);
  int resident = 0;
  MKG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, fwd_fn, kFwdWarps * 32, 0));
  // one wave of resident blocks, split evenly over the column chunks
  const int blocks_per_chunk = grid_for(adj->num_pull_tasks, kFwdWarps,
                                        (int)((int64_t)num_sms() * (resident > 0 ? resident : 1) / nfch) + 1);
  for (int64_t h = 0; h < q.hops; ++h) {
    float* y = S.y(h);
    if (ix && ix->num_slots > 0) {
      const int64_t take_blocks = ix->num_slots * ((q.BLP + kTakeCols - 1) / kTakeCols);
      cap_take_kernel<<<(unsigned)(take_blocks < (int64_t)pb * 8 ? take_blocks : (int64_t)pb * 8), kTakeCols, 0, st>>>(
          make_dir(g->ori), make_dir(g->inv), ix->slot_entity, ix->slot_dir, ix->slot_group, ix->num_slots, q, S.wt(h),
          S.act(h), S.take(h), err);
      MKG_LAUNCHED("cap_take_kernel");
    }
    dim3 grid(blocks_per_chunk, (unsigned)nfch);
    if (p->fwd_events) MKG_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(p->fwd_events[2 * h]), st));
    {
      const int4* tk = reinterpret_cast<const int4*>(adj->pull_tasks);
      const int64_t nt = adj->num_pull_tasks;
      float* ds = max_mode ? nullptr : S.d(h);
      uint8_t* yh = max_mode ? nullptr : S.yact(h);
      int32_t* qu = S.queue() + h * q.nch * kQueueStride;
      const uint8_t* tk_h = ix ? S.take(h) : nullptr;
#define MKG_FWD_PULL(M, V, C) \
  fwd_pull_kernel<M, V, C><<<grid, kFwdWarps * 32, 0, st>>>(tk, nt, adj->pull, q, S.wt(h), S.x(h), S.act(h), y, ds, \
                                                           yh, qu, pull_cap, tk_h, err)
      if (ix) {
        if (max_mode && vec == 2) MKG_FWD_PULL(true, 2, true);
        else if (max_mode) MKG_FWD_PULL(true, 1, true);
        else if (vec == 2) MKG_FWD_PULL(false, 2, true);
        else MKG_FWD_PULL(false, 1, true);
      } else {
        if (max_mode && vec == 2) MKG_FWD_PULL(true, 2, false);
        else if (max_mode) MKG_FWD_PULL(true, 1, false);
        else if (vec == 2) MKG_FWD_PULL(false, 2, false);
        else MKG_FWD_PULL(false, 1, false);
      }
#undef MKG_FWD_PULL
    }
    MKG_LAUNCHED("fwd_pull_kernel");
    if (p->fwd_events) MKG_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(p->fwd_events[2 * h + 1]), st));
    if (max_mode) {
      CUtensorMap ymap;
      rc = make_rows_map(&ymap, y, q.E, q.BLP);
      if (rc) return rc;
      sequential_colsum_kernel<<<(unsigned)((q.BLP + 31) / 32), 64, 0, st>>>(ymap, q, S.d(h), err);
      MKG_LAUNCHED("sequential_colsum_kernel");
      if (h + 1 < q.hops) {
        normalize_plain_kernel<<<pb, 256, 0, st>>>(y, S.d(h), q, S.x(h + 1), S.act(h + 1), adj->push_ptr, capdeg,
                                                   S.msgs() + h + 1);
        MKG_LAUNCHED("normalize_plain_kernel");
      }
    } else {
      normalize_mass_kernel<<<pb, 256, 0, st>>>(y, S.d(h), q, p->state_threshold, h + 1 == q.hops, S.x(h + 1),
                                                S.act(h + 1), S.yact(h), adj->push_ptr, capdeg, S.msgs() + h + 1);
      MKG_LAUNCHED("normalize_mass_kernel");
    }
  }
  dim3 tgrid((unsigned)((q.E + 31) / 32), (unsigned)((q.B + 31) / 32));
  if (max_mode)
    rows_to_queries_kernel<true><<<tgrid, dim3(32, 8), 0, st>>>(S.y(q.hops - 1), S.d(q.hops - 1), q, out);
  else
    rows_to_queries_kernel<false><<<tgrid, dim3(32, 8), 0, st>>>(S.x(q.hops), nullptr, q, out);
  MKG_LAUNCHED("rows_to_queries_kernel");
  if (messages_out) MKG_CUDA(cudaMemcpyAsync(messages_out, S.msgs(), 8 * (size_t)q.hops, cudaMemcpyDeviceToDevice, st));
  return MKG_OK;
}

int proof_forward(const mkg_graph* g, const mkg_adjacency* adj, const int64_t* heads, const float* w_hops,
                  const mkg_proof_params* p, void* ws, size_t ws_bytes, float* out, int64_t* messages_out,
                  unsigned* err, cudaStream_t st) {
  return run_forward(g, adj, heads, w_hops, p, false, ws, ws_bytes, out, messages_out, err, st);
}

int proof_backward(const mkg_graph* g, const mkg_adjacency* adj, const float* w_hops, const mkg_proof_params* p,
                   const mkg_edge_factor* ef, const float* grad_out, float* grad_w_hops, float* grad_edge, void* ws,
                   size_t ws_bytes, unsigned* err, cudaStream_t st) {
  int rc = check_proof(g, adj, p);
  if (rc) return rc;
  MKG_REQUIRE(grad_out && grad_w_hops && ef, "proof_backward: null argument");
  (void)w_hops;  // the transposed weights of the forward are still in the workspace
  const ProofDims q = proof_dims(*p);
  Slab S{static_cast<char*>(ws), proof_layout(q), q};
  MKG_REQUIRE(ws && ws_bytes >= S.lay.total, "proof_backward: workspace too small");
  const size_t slab = 4 * (size_t)q.E * q.BLP;
  const int pb = persistent_blocks(4);
  EdgeFactor f = make_factor(*ef);
  backward_setup_kernel<<<pb, 256, 0, st>>>(q, grad_edge, g->num_facts, S.s(0), S.queue() + q.hops * q.nch * kQueueStride,
                                            q.hops * q.nch * kQueueStride, S.dwt());
  MKG_LAUNCHED("backward_setup_kernel");
  float* dx_cur = S.dxa();
  float* dx_next = S.dxb();
  dim3 sgrid((unsigned)((q.E + 32 * kSeedTiles - 1) / (32 * kSeedTiles)), (unsigned)((q.B + 31) / 32));
  seed_grad_kernel<<<sgrid, 256, 0, st>>>(grad_out, S.x(q.hops), S.y(q.hops - 1), q, dx_cur, S.s(q.hops - 1));
  MKG_LAUNCHED("seed_grad_kernel");
  const mkg_cap_index* ix = q.cap >= 0 ? p->cap_index : nullptr;
  const int2* push_cap = ix ? reinterpret_cast<const int2*>(ix->push_cap) : nullptr;
  // fp64 rule-weight partials wherever they keep the fp32 variant's blocks per SM (few relation
  // channels); fp32 where the doubled shared memory would cost occupancy (measured on the
  // 51-relation workload: 2 instead of 4 blocks per SM, 1.45 -> 1.83 ms per step)
  const void* fn32 = ix ? (const void*)bwd_pull_kernel<true, float> : (const void*)bwd_pull_kernel<false, float>;
  const void* fn64 = ix ? (const void*)bwd_pull_kernel<true, double> : (const void*)bwd_pull_kernel<false, double>;
  int occ32 = 0, occ64 = 0;
  rc = set_smem(fn32, bwd_smem(q, false));
  if (rc) return rc;
  MKG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ32, fn32, kBwdWarps * 32, bwd_smem(q, false)));
  if (bwd_smem(q, true) <= kBwdSmemMax) {
    rc = set_smem(fn64, bwd_smem(q, true));
    if (rc) return rc;
    MKG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ64, fn64, kBwdWarps * 32, bwd_smem(q, true)));
  }
  const bool f64 = occ64 >= 1 && occ64 >= occ32;
  const void* bwd_fn = f64 ? fn64 : fn32;
  const size_t sm = bwd_smem(q, f64);
  const int resident = f64 ? occ64 : occ32;
  const int blocks_per_chunk = grid_for(adj->num_push_tasks, kBwdWarps,
                                        (int)((int64_t)num_sms() * (resident > 0 ? resident : 1) / q.nch) + 1);
  for (int64_t h = q.hops - 1; h >= 0; --h) {
    // dY_h from dX_{h+1}
    normalize_mass_backward_kernel<<<pb, 256, 0, st>>>(dx_cur, S.y(h), S.d(h), S.s(h), S.yact(h), q, S.dy(),
                                                       reinterpret_cast<const int4*>(adj->push_tasks),
                                                       adj->num_push_tasks, dx_next);
    MKG_LAUNCHED("normalize_mass_backward_kernel");
    (void)slab;
    dim3 grid(blocks_per_chunk, (unsigned)q.nch);
    if (p->bwd_events) MKG_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(p->bwd_events[2 * h]), st));
    {
      const int4* tk = reinterpret_cast<const int4*>(adj->push_tasks);
      int32_t* qu = S.queue() + (q.hops + h) * q.nch * kQueueStride;
      auto launch = [&](auto kernel, const int2* rcap, const uint8_t* take) {
        kernel<<<grid, kBwdWarps * 32, sm, st>>>(
            tk, adj->num_push_tasks, adj->push, q, S.wt(h), S.x(h), S.act(h), S.yact(h), S.dy(),
            h > 0 ? S.y(h - 1) : nullptr, dx_next, S.dwt(), h > 0 ? S.s(h - 1) : nullptr, grad_edge, g->num_facts, f,
            qu, rcap, take, err);
      };
      if (ix) {
        if (f64) launch(bwd_pull_kernel<true, double>, push_cap, S.take(h));
        else launch(bwd_pull_kernel<true, float>, push_cap, S.take(h));
      } else {
        if (f64) launch(bwd_pull_kernel<false, double>, nullptr, nullptr);
        else launch(bwd_pull_kernel<false, float>, nullptr, nullptr);
      }
    }
    MKG_LAUNCHED("bwd_pull_kernel");
    if (p->bwd_events) MKG_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(p->bwd_events[2 * h + 1]), st));
    untranspose_dw_kernel<<<grid_for(q.BL * q.n, 256, pb), 256, 0, st>>>(S.dwt(), q, h, grad_w_hops);
    MKG_LAUNCHED("untranspose_dw_kernel");
    float* t = dx_cur; dx_cur = dx_next; dx_next = t;
  }
  return MKG_OK;
}

namespace {
__global__ void row_activity_kernel(const uint8_t* __restrict__ act, ProofDims q, uint8_t* __restrict__ flags) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < q.E; e += (int64_t)gridDim.x * blockDim.x) {
    uint8_t any = 0;
    for (int64_t c = 0; c < q.nch; ++c) any |= act[e * q.nch + c];
    flags[e] = any ? 1 : 0;
  }
}
}  // namespace

int proof_row_activity(const mkg_proof_params* p, const void* ws, size_t ws_bytes, int64_t h, uint8_t* flags,
                       cudaStream_t st) {
  MKG_REQUIRE(p && ws && flags, "proof_row_activity: null argument");
  const ProofDims q = proof_dims(*p);
  MKG_REQUIRE(h >= 0 && h <= q.hops, "proof_row_activity: hop out of range");
  Slab S{static_cast<char*>(const_cast<void*>(ws)), proof_layout(q), q};
  MKG_REQUIRE(ws_bytes >= S.lay.total, "proof_row_activity: workspace too small");
  row_activity_kernel<<<grid_for(q.E, 256, persistent_blocks(4)), 256, 0, st>>>(S.act(h), q, flags);
  MKG_LAUNCHED("row_activity_kernel");
  return MKG_OK;
}

size_t decode_workspace_bytes(const mkg_proof_params* p, int64_t topk) {
  (void)topk;
  return proof_layout(proof_dims(*p)).total + 256;
}

int proof_decode_max(const mkg_graph* g, const mkg_adjacency* adj, const int64_t* heads, const float* w_hops,
                     const mkg_proof_params* p, int64_t topk, float* out_scores, int64_t* tails, float* scores,
                     int64_t* counts, void* ws, size_t ws_bytes, unsigned* err, cudaStream_t st) {
  MKG_REQUIRE(topk >= 1 && topk <= kTopkMax, "decode: topk must lie in [1, %d]", kTopkMax);
  MKG_REQUIRE(tails && scores && counts, "decode: null output");
  int rc = run_forward(g, adj, heads, w_hops, p, true, ws, ws_bytes, out_scores, nullptr, err, st);
  if (rc) return rc;
  topk_rows_kernel<<<(unsigned)p->B, kTopkThreads, 0, st>>>(DenseTopkRows{out_scores, p->E}, topk, tails, scores,
                                                             counts);
  MKG_LAUNCHED("topk_rows_kernel");
  return MKG_OK;
}

namespace {
// One thread per segment: a sequential fp32 chain in index order.
// One warp per segment: the warp stages kOrdChunk values at a time through shared memory with
// coalesced loads, and lane 0 adds them one by one in index order (the sum is a single fp32
// chain, as a sequential CPU loop forms it).  The loads of the next chunk are issued before lane
// 0 starts on the current one, so memory latency overlaps the dependent adds.
constexpr int kOrdWarps = 4;
constexpr int kOrdPerLane = 32;
constexpr int kOrdChunk = 32 * kOrdPerLane;

__global__ void __launch_bounds__(kOrdWarps * 32) segment_sum_ordered_kernel(const int64_t* __restrict__ seg_ptr,
                                                                           int64_t nseg,
                                                                           const float* __restrict__ values,
                                                                           float* __restrict__ out) {
  __shared__ __align__(16) float buf[kOrdWarps][kOrdChunk];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float* sb = buf[w];
  for (int64_t s = blockIdx.x * (int64_t)kOrdWarps + w; s < nseg; s += (int64_t)gridDim.x * kOrdWarps) {
    const int64_t b = seg_ptr[s], e = seg_ptr[s + 1];
    float r[kOrdPerLane];
#pragma unroll
    for (int k = 0; k < kOrdPerLane; ++k) {
      const int64_t i = b + k * 32 + lane;
      r[k] = i < e ? values[i] : 0.0f;
    }
    float acc = 0.0f;
    for (int64_t c0 = b; c0 < e; c0 += kOrdChunk) {
#pragma unroll
      for (int k = 0; k < kOrdPerLane; ++k) sb[k * 32 + lane] = r[k];
      __syncwarp();
      const int64_t c1 = c0 + kOrdChunk;
      if (c1 < e) {
#pragma unroll
        for (int k = 0; k < kOrdPerLane; ++k) {
          const int64_t i = c1 + k * 32 + lane;
          r[k] = i < e ? values[i] : 0.0f;
        }
      }
      if (lane == 0) {
        const int m = static_cast<int>(e - c0 < kOrdChunk ? e - c0 : kOrdChunk);
        const int m4 = m & ~3;
        for (int j = 0; j < m4; j += 4) {
          const float4 v = *reinterpret_cast<const float4*>(sb + j);
          acc = __fadd_rn(acc, v.x);
          acc = __fadd_rn(acc, v.y);
          acc = __fadd_rn(acc, v.z);
          acc = __fadd_rn(acc, v.w);
        }
        for (int j = m4; j < m; ++j) acc = __fadd_rn(acc, sb[j]);
      }
      __syncwarp();
    }
    if (lane == 0) out[s] = acc;
  }
}
// One block per segment: strided partial sums, then a block reduction.
__global__ void __launch_bounds__(256) segment_sum_kernel(const int64_t* __restrict__ seg_ptr, int64_t nseg,
                                                          const float* __restrict__ values, float* __restrict__ out) {
  typedef cub::BlockReduce<float, 256> Reduce;
  __shared__ typename Reduce::TempStorage tmp;
  for (int64_t s = blockIdx.x; s < nseg; s += gridDim.x) {
    const int64_t b = seg_ptr[s], e = seg_ptr[s + 1];
    float acc = 0.0f;
    for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x) acc += values[i];
    const float tot = Reduce(tmp).Sum(acc);
    if (threadIdx.x == 0) out[s] = tot;
    __syncthreads();
  }
}
}  // namespace

int segment_sum(const int64_t* seg_ptr, int64_t nseg, const float* values, float* out, cudaStream_t st) {
  MKG_REQUIRE(nseg >= 0, "segment_sum: negative segment count");
  if (nseg == 0) return MKG_OK;
  MKG_REQUIRE(seg_ptr && values && out, "segment_sum: null argument");
  segment_sum_kernel<<<grid_for(nseg, 1, persistent_blocks(8)), 256, 0, st>>>(seg_ptr, nseg, values, out);
  MKG_LAUNCHED("segment_sum_kernel");
  return MKG_OK;
}

int segment_sum_ordered(const int64_t* seg_ptr, int64_t nseg, const float* values, float* out, cudaStream_t st) {
  MKG_REQUIRE(nseg >= 0, "segment_sum_ordered: negative segment count");
  if (nseg == 0) return MKG_OK;
  MKG_REQUIRE(seg_ptr && values && out, "segment_sum_ordered: null argument");
  segment_sum_ordered_kernel<<<grid_for(nseg, kOrdWarps, persistent_blocks(16)), kOrdWarps * 32, 0, st>>>(
      seg_ptr, nseg, values, out);
  MKG_LAUNCHED("segment_sum_ordered_kernel");
  return MKG_OK;
}

int decode_topk(const float* raw, int64_t B, int64_t E, int64_t topk, int64_t* tails, float* scores,
                int64_t* counts, cudaStream_t st) {
  MKG_REQUIRE(raw && tails && scores && counts, "decode_topk: null argument");
  MKG_REQUIRE(topk >= 1 && topk <= kTopkMax, "decode_topk: topk must lie in [1, %d]", kTopkMax);
  MKG_REQUIRE(B >= 1 && E >= 1 && E < (int64_t(1) << 32) - 1, "decode_topk: bad sizes");
  topk_rows_kernel<<<(unsigned)B, kTopkThreads, 0, st>>>(DenseTopkRows{raw, E}, topk, tails, scores, counts);
  MKG_LAUNCHED("topk_rows_kernel");
  return MKG_OK;
}

size_t sparse_topk_workspace_bytes(int64_t nnz) { return nnz > 0 ? 8 * (size_t)nnz : 0; }

int sparse_topk(const int64_t* keys, const float* vals, int64_t nnz, int64_t B, int64_t E, int64_t topk,
                int64_t* tails, float* scores, int64_t* counts, void* ws, size_t ws_bytes, cudaStream_t st) {
  MKG_REQUIRE(tails && scores && counts && (nnz == 0 || (keys && vals && ws)), "sparse_topk: null argument");
  MKG_REQUIRE(topk >= 1 && topk <= kTopkMax, "sparse_topk: topk must lie in [1, %d]", kTopkMax);
  MKG_REQUIRE(nnz >= 0 && B >= 1 && E >= 1 && E < (int64_t(1) << 32) - 1 && B <= (int64_t(1) << 62) / E,
              "sparse_topk: bad sizes");
  MKG_REQUIRE(ws_bytes >= sparse_topk_workspace_bytes(nnz), "sparse_topk: workspace too small");
  auto* cand = static_cast<unsigned long long*>(ws);
  if (nnz > 0) {
    sparse_candidate_keys_kernel<<<grid_for(nnz, 256, persistent_blocks(8)), 256, 0, st>>>(keys, vals, nnz, E, cand);
    MKG_LAUNCHED("sparse_candidate_keys_kernel");
  }
  topk_rows_kernel<<<(unsigned)B, kTopkThreads, 0, st>>>(SparseTopkRows{keys, cand, nnz, E}, topk, tails, scores,
                                                          counts);
  MKG_LAUNCHED("topk_rows_kernel");
  return MKG_OK;
}

}  // namespace mkg
