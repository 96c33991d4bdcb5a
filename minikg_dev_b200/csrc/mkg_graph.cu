// Graph build on the device: the reference CSR pair (stable radix sort), ind2ptr, the
// per-fact endpoint table and the merged pull / push neighbour lists of the fused engine.
#include <cub/cub.cuh>

#include "mkg_common.cuh"

namespace mkg {
namespace {

__global__ void make_keys_kernel(const int32_t* __restrict__ row, const int32_t* __restrict__ rel,
                                 const int32_t* __restrict__ col, int64_t T, int64_t E, int64_t R,
                                 unsigned long long* __restrict__ keys, int32_t* __restrict__ ids,
                                 unsigned* err) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < T;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = row[i], c = col[i], q = rel[i];
    if (r < 0 || r >= E || c < 0 || c >= E) { raise_flag(err, MKG_DEV_BAD_COL); r = 0; }
    if (q < 0 || q >= R) { raise_flag(err, MKG_DEV_BAD_REL); q = 0; }
    keys[i] = static_cast<unsigned long long>(r) * static_cast<unsigned long long>(R) +
              static_cast<unsigned long long>(q);
    ids[i] = static_cast<int32_t>(i);
  }
}

// Gathers the sorted arrays and flags the first position of every (row, rel) group.
__global__ void gather_sorted_kernel(const unsigned long long* __restrict__ skeys,
                                     const int32_t* __restrict__ order, const int32_t* __restrict__ col,
                                     const int32_t* __restrict__ rel, int64_t T,
                                     int32_t* __restrict__ col_out, int16_t* __restrict__ rel_out,
                                     int32_t* __restrict__ group_flag) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < T;
       p += (int64_t)gridDim.x * blockDim.x) {
    int32_t f = order[p];
    col_out[p] = col[f];
    rel_out[p] = static_cast<int16_t>(rel[f]);
    group_flag[p] = (p == 0 || skeys[p] != skeys[p - 1]) ? 1 : 0;
  }
}

// row_ptr[r] = first sorted position whose row is >= r (boundary fill, O(E + T)).
__global__ void row_ptr_kernel(const unsigned long long* __restrict__ skeys, int64_t T, int64_t E,
                               int64_t R, int32_t* __restrict__ row_ptr) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p <= T;
       p += (int64_t)gridDim.x * blockDim.x) {
    int64_t cur = p < T ? static_cast<int64_t>(skeys[p] / static_cast<unsigned long long>(R)) : E;
    int64_t prev = p > 0 ? static_cast<int64_t>(skeys[p - 1] / static_cast<unsigned long long>(R)) : -1;
    for (int64_t r = prev + 1; r <= cur && r <= E; ++r) row_ptr[r] = static_cast<int32_t>(p);
  }
}

// Group metadata from the inclusive scan of the group flags.
__global__ void groups_kernel(const unsigned long long* __restrict__ skeys,
                              const int32_t* __restrict__ gflag, const int32_t* __restrict__ gscan,
                              int64_t T, int64_t R, int16_t* __restrict__ group_rel,
                              int32_t* __restrict__ group_start, int32_t* __restrict__ group_count,
                              int32_t* __restrict__ group_row) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < T;
       p += (int64_t)gridDim.x * blockDim.x) {
    if (!gflag[p]) continue;
    int32_t gi = gscan[p] - 1;
    group_rel[gi] = static_cast<int16_t>(skeys[p] % static_cast<unsigned long long>(R));
    group_start[gi] = static_cast<int32_t>(p);
    group_row[gi] = static_cast<int32_t>(skeys[p] / static_cast<unsigned long long>(R));
    // count = distance to the next group start
    int64_t q = p + 1;
    while (q < T && !gflag[q]) ++q;
    group_count[gi] = static_cast<int32_t>(q - p);
  }
}

__global__ void store_group_count_kernel(const int32_t* __restrict__ gscan, int64_t T,
                                         int64_t* __restrict__ out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *out = T > 0 ? gscan[T - 1] : 0;
}

struct CsrScratch {
  unsigned long long* keys_in;
  unsigned long long* keys_out;
  int32_t* ids;
  int32_t* gflag;
  int32_t* gscan;
  int32_t* group_row;
  void* cub_temp;
  size_t cub_bytes;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

size_t cub_bytes_for(int64_t T, int end_bit) {
  size_t a = 0, b = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, a, (unsigned long long*)nullptr, (unsigned long long*)nullptr,
                                  (int32_t*)nullptr, (int32_t*)nullptr, (int)T, 0, end_bit);
  cub::DeviceScan::InclusiveSum(nullptr, b, (int32_t*)nullptr, (int32_t*)nullptr, (int)T);
  return a > b ? a : b;
}

int key_bits(int64_t E, int64_t R) {
  unsigned long long mx = static_cast<unsigned long long>(E) * static_cast<unsigned long long>(R);
  int bits = 1;
  while (bits < 64 && (1ull << bits) <= mx) ++bits;
  return bits;
}

CsrScratch carve(void* ws, int64_t T, int64_t E, int64_t R) {
  CsrScratch s;
  char* p = static_cast<char*>(ws);
  s.keys_in = reinterpret_cast<unsigned long long*>(p); p += align256(8 * T);
  s.keys_out = reinterpret_cast<unsigned long long*>(p); p += align256(8 * T);
  s.ids = reinterpret_cast<int32_t*>(p); p += align256(4 * T);
  s.gflag = reinterpret_cast<int32_t*>(p); p += align256(4 * T);
  s.gscan = reinterpret_cast<int32_t*>(p); p += align256(4 * T);
  s.group_row = reinterpret_cast<int32_t*>(p); p += align256(4 * T);
  s.cub_temp = p;
  s.cub_bytes = cub_bytes_for(T, key_bits(E, R));
  return s;
}

int build_direction(const int32_t* row, const int32_t* rel, const int32_t* col, int64_t T, int64_t E,
                    int64_t R, mkg_csr_dir_out out, int64_t* num_groups, CsrScratch& s,
                    unsigned* err, cudaStream_t st) {
  const int blocks = persistent_blocks(4), threads = 256;
  make_keys_kernel<<<blocks, threads, 0, st>>>(row, rel, col, T, E, R, s.keys_in, s.ids, err);
  MKG_LAUNCHED("make_keys_kernel");
  size_t bytes = s.cub_bytes;
  MKG_CUDA(cub::DeviceRadixSort::SortPairs(s.cub_temp, bytes, s.keys_in, s.keys_out, s.ids, out.order,
                                           (int)T, 0, key_bits(E, R), st));
  gather_sorted_kernel<<<blocks, threads, 0, st>>>(s.keys_out, out.order, col, rel, T, out.col_ind,
                                                   out.r_ind, s.gflag);
  MKG_LAUNCHED("gather_sorted_kernel");
  row_ptr_kernel<<<blocks, threads, 0, st>>>(s.keys_out, T, E, R, out.row_ptr);
  MKG_LAUNCHED("row_ptr_kernel");
  bytes = s.cub_bytes;
  MKG_CUDA(cub::DeviceScan::InclusiveSum(s.cub_temp, bytes, s.gflag, s.gscan, (int)T, st));
  groups_kernel<<<blocks, threads, 0, st>>>(s.keys_out, s.gflag, s.gscan, T, R, out.group_rel,
                                            out.group_edge_start, out.group_edge_count, s.group_row);
  MKG_LAUNCHED("groups_kernel");
  store_group_count_kernel<<<1, 32, 0, st>>>(s.gscan, T, num_groups);
  MKG_LAUNCHED("store_group_count_kernel");
  // row_group_ptr needs the group count, which only the device knows: the caller launches
  // group_ptr_from_count_kernel, which reads it from num_groups.
  return MKG_OK;
}

__global__ void group_ptr_from_count_kernel(const int32_t* __restrict__ group_row,
                                            const int64_t* __restrict__ num_groups, int64_t E,
                                            int32_t* __restrict__ group_ptr) {
  const int64_t G = *num_groups;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g <= G;
       g += (int64_t)gridDim.x * blockDim.x) {
    int64_t cur = g < G ? group_row[g] : E;
    int64_t prev = g > 0 ? group_row[g - 1] : -1;
    for (int64_t r = prev + 1; r <= cur && r <= E; ++r) group_ptr[r] = static_cast<int32_t>(g);
  }
}

__global__ void ind2ptr_count_kernel(const int64_t* __restrict__ index, int64_t n, int64_t size,
                                     int64_t* __restrict__ ptr, unsigned* err) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = index[i];
    if (r < 0 || r >= size) { raise_flag(err, MKG_DEV_BAD_ENTRY); continue; }
    atomicAdd(reinterpret_cast<unsigned long long*>(ptr + r + 1), 1ull);
  }
}

__device__ __forceinline__ int64_t row_of_position(const int32_t* __restrict__ row_ptr, int64_t E,
                                                   int64_t p) {
  int64_t lo = 0, hi = E;  // invariant: row_ptr[lo] <= p < row_ptr[hi]
  while (hi - lo > 1) {
    int64_t mid = (lo + hi) >> 1;
    if (row_ptr[mid] <= p) lo = mid; else hi = mid;
  }
  return lo;
}

__global__ void fact_table_kernel(DirCSR ori, int64_t E, int64_t T, int32_t* __restrict__ head,
                                  int32_t* __restrict__ tail, int16_t* __restrict__ rel, unsigned* err) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < T;
       p += (int64_t)gridDim.x * blockDim.x) {
    int64_t f = ori.order[p];
    if (f < 0 || f >= T) { raise_flag(err, MKG_DEV_BAD_FACT); continue; }
    head[f] = static_cast<int32_t>(row_of_position(ori.row_ptr, E, p));
    tail[f] = ori.col[p];
    rel[f] = ori.rel[p];
  }
}

__global__ void adjacency_ptr_kernel(const int32_t* __restrict__ a_ptr, const int32_t* __restrict__ b_ptr,
                                     int64_t E, int32_t* __restrict__ out) {
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r <= E;
       r += (int64_t)gridDim.x * blockDim.x)
    out[r] = a_ptr[r] + b_ptr[r];
}

// Places the CSR positions of `src` into the merged rows: record index =
// merged_ptr[row] + first_part_len(row) * second + (p - src.row_ptr[row]).
__global__ void adjacency_fill_kernel(DirCSR src, const int32_t* __restrict__ other_row_ptr, int64_t E,
                                      int64_t T, int64_t chan_off, int second,
                                      const int32_t* __restrict__ merged_ptr,
                                      mkg_adj_edge* __restrict__ out, unsigned* err) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < T;
       p += (int64_t)gridDim.x * blockDim.x) {
    int64_t row = row_of_position(src.row_ptr, E, p);
    int64_t base = merged_ptr[row];
    if (second) base += other_row_ptr[row + 1] - other_row_ptr[row];
    int64_t idx = base + (p - src.row_ptr[row]);
    int32_t nbr = src.col[p];
    int32_t fact = src.order[p];
    if (nbr < 0 || nbr >= E) raise_flag(err, MKG_DEV_BAD_COL);
    if (fact < 0 || fact >= T) raise_flag(err, MKG_DEV_BAD_FACT);
    mkg_adj_edge rec;
    rec.nbr = nbr;
    rec.channel = static_cast<int32_t>(chan_off + src.rel[p]);
    rec.fact = fact;
    rec.factor = 1.0f;
    out[idx] = rec;
  }
}

constexpr int kTaskSeg = 64;  // records per task of the fused engine

__global__ void task_count_kernel(const int32_t* __restrict__ ptr, int64_t E, int32_t* __restrict__ nt) {
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r <= E;
       r += (int64_t)gridDim.x * blockDim.x) {
    if (r == E) { nt[r] = 0; continue; }
    const int64_t deg = ptr[r + 1] - ptr[r];
    nt[r] = deg <= kTaskSeg ? 1 : static_cast<int32_t>((deg + kTaskSeg - 1) / kTaskSeg);
  }
}

__global__ void task_fill_kernel(const int32_t* __restrict__ ptr, const int32_t* __restrict__ nt,
                                 const int32_t* __restrict__ offs, int64_t E, int4* __restrict__ tasks,
                                 int64_t* __restrict__ total) {
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < E;
       r += (int64_t)gridDim.x * blockDim.x) {
    const int32_t n = nt[r], o = offs[r], p0 = ptr[r], p1 = ptr[r + 1];
    for (int32_t j = 0; j < n; ++j) {
      const int32_t b = p0 + j * kTaskSeg;
      const int32_t e = min(b + kTaskSeg, p1);
      tasks[o + j] = make_int4(static_cast<int32_t>(r), b, e, (j == 0 ? 1 : 0) | (n > 1 ? 2 : 0));
    }
    if (r == E - 1) *total = o + n;
  }
}

// (Four records per thread with their loads issued together measured slower: 131 against 116 us
// per 10 M-record launch.)
__global__ void adjacency_factor_kernel(mkg_adj_edge* __restrict__ recs, int64_t count, int64_t T, EdgeFactor f) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t fact = recs[i].fact;
    recs[i].factor = (fact >= 0 && fact < T) ? f(fact) : 0.0f;
  }
}

// ---------------------------------------------------------------- edge-cap index
// flag[dir * E + e] = row e of direction dir is longer than the cap; ngrp = its group count
// (0 when not capped); capdeg[e] = messages an active entry of e sends under the cap.
// flag and ngrp carry one extra trailing 0 so that their exclusive scans end in the totals.
__global__ void cap_rows_kernel(DirCSR ori, DirCSR inv, int64_t E, int64_t cap, int32_t* __restrict__ flag,
                                int32_t* __restrict__ ngrp, int32_t* __restrict__ capdeg) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e <= E; e += (int64_t)gridDim.x * blockDim.x) {
    if (e == E) { flag[2 * E] = 0; ngrp[2 * E] = 0; continue; }
    const int64_t dori = ori.row_ptr[e + 1] - ori.row_ptr[e], dinv = inv.row_ptr[e + 1] - inv.row_ptr[e];
    const bool fo = dori > cap, fi = dinv > cap;
    flag[e] = fo;
    flag[E + e] = fi;
    ngrp[e] = fo ? ori.group_ptr[e + 1] - ori.group_ptr[e] : 0;
    ngrp[E + e] = fi ? inv.group_ptr[e + 1] - inv.group_ptr[e] : 0;
    if (capdeg) capdeg[e] = static_cast<int32_t>((dori < cap ? dori : cap) + (dinv < cap ? dinv : cap));
  }
}

__global__ void cap_sizes_kernel(const int32_t* __restrict__ sidx, const int32_t* __restrict__ gbase, int64_t E,
                                 int64_t* __restrict__ sizes) {
  sizes[0] = sidx[2 * E];
  sizes[1] = gbase[2 * E];
}

__global__ void cap_slots_kernel(const int32_t* __restrict__ flag, const int32_t* __restrict__ sidx,
                                 const int32_t* __restrict__ gbase, int64_t E, int64_t num_slots,
                                 int32_t* __restrict__ slot_entity, int32_t* __restrict__ slot_dir,
                                 int32_t* __restrict__ slot_group, unsigned* err) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < 2 * E; i += (int64_t)gridDim.x * blockDim.x) {
    if (!flag[i]) continue;
    const int64_t si = sidx[i];
    if (si < 0 || si >= num_slots) { raise_flag(err, MKG_DEV_BAD_ENTRY); continue; }
    slot_entity[si] = static_cast<int32_t>(i % E);
    slot_dir[si] = static_cast<int32_t>(i / E);
    slot_group[si] = gbase[i];
  }
}

// Per CSR position p of direction dir (row = the sending entity): fact_cap[dir][fact] =
// (take-table row of p's relation group, p's position inside the group), or (-1, 0) when the
// row is not capped.
__global__ void cap_fact_kernel(DirCSR d, int dir, int64_t E, int64_t T, const int32_t* __restrict__ flag,
                                const int32_t* __restrict__ gbase, int2* __restrict__ fact_cap, unsigned* err) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < T; p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t f = d.order[p];
    if (f < 0 || f >= T) { raise_flag(err, MKG_DEV_BAD_FACT); continue; }
    const int64_t row = row_of_position(d.row_ptr, E, p);
    int2 out = make_int2(-1, 0);
    if (flag[dir * E + row]) {
      int64_t lo = d.group_ptr[row], hi = d.group_ptr[row + 1];  // group_start[lo] <= p
      while (hi - lo > 1) {
        const int64_t mid = (lo + hi) >> 1;
        if (d.group_start[mid] <= p) lo = mid; else hi = mid;
      }
      out = make_int2(static_cast<int32_t>(gbase[dir * E + row] + (lo - d.group_ptr[row])),
                      static_cast<int32_t>(p - d.group_start[lo]));
    }
    fact_cap[dir * T + f] = out;
  }
}

// Per record: the entry of its (direction, fact); channel < R is an ori message of the sender.
__global__ void cap_records_kernel(const mkg_adj_edge* __restrict__ recs, int64_t count, int64_t T, int64_t R,
                                   const int2* __restrict__ fact_cap, int2* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    const mkg_adj_edge r = recs[i];
    const int dir = r.channel < R ? 0 : 1;
    out[i] = (r.fact >= 0 && r.fact < T) ? fact_cap[dir * T + r.fact] : make_int2(-1, 0);
  }
}

}  // namespace

size_t csr_build_workspace_bytes(int64_t T, int64_t E, int64_t R) {
  return 6 * align256(8 * (size_t)T) + align256(cub_bytes_for(T, key_bits(E, R))) + 256;
}

int csr_build(const int32_t* head, const int32_t* rel, const int32_t* tail, int64_t T, int64_t E,
              int64_t R, mkg_csr_dir_out ori, mkg_csr_dir_out inv, int64_t* num_groups, void* ws,
              size_t ws_bytes, unsigned* err, cudaStream_t st) {
  MKG_REQUIRE(T >= 1 && T < (int64_t(1) << 31), "csr_build: num_facts %lld out of range", (long long)T);
  MKG_REQUIRE(E >= 1 && E < (int64_t(1) << 31) && R >= 1 && R <= 32767,
              "csr_build: entity / relation count out of range (E=%lld R=%lld)", (long long)E, (long long)R);
  MKG_REQUIRE(ws_bytes >= csr_build_workspace_bytes(T, E, R), "csr_build: workspace too small");
  CsrScratch s = carve(ws, T, E, R);
  int rc = build_direction(head, rel, tail, T, E, R, ori, num_groups, s, err, st);
  if (rc) return rc;
  group_ptr_from_count_kernel<<<persistent_blocks(4), 256, 0, st>>>(s.group_row, num_groups, E,
                                                                     ori.row_group_ptr);
  MKG_LAUNCHED("group_ptr_from_count_kernel");
  rc = build_direction(tail, rel, head, T, E, R, inv, num_groups + 1, s, err, st);
  if (rc) return rc;
  group_ptr_from_count_kernel<<<persistent_blocks(4), 256, 0, st>>>(s.group_row, num_groups + 1, E,
                                                                     inv.row_group_ptr);
  MKG_LAUNCHED("group_ptr_from_count_kernel");
  return MKG_OK;
}

size_t ind2ptr_workspace_bytes(int64_t size) {
  size_t b = 0;
  cub::DeviceScan::InclusiveSum(nullptr, b, (int64_t*)nullptr, (int64_t*)nullptr, (int)size);
  return align256(8 * (size_t)(size + 1)) + align256(b) + 256;
}

int ind2ptr(const int64_t* index, int64_t n, int64_t size, int64_t* ptr, void* ws, size_t ws_bytes,
            unsigned* err, cudaStream_t st) {
  MKG_REQUIRE(size >= 0 && size < (int64_t(1) << 31) && n >= 0, "ind2ptr: bad sizes");
  MKG_REQUIRE(ws_bytes >= ind2ptr_workspace_bytes(size), "ind2ptr: workspace too small");
  // counts land in cnt[1..size]; the scan writes ptr[1..size]; ptr[0] = 0
  int64_t* cnt = static_cast<int64_t*>(ws);
  void* temp = static_cast<char*>(ws) + align256(8 * (size_t)(size + 1));
  MKG_CUDA(cudaMemsetAsync(cnt, 0, sizeof(int64_t) * (size + 1), st));
  MKG_CUDA(cudaMemsetAsync(ptr, 0, sizeof(int64_t), st));
  if (n > 0) {
    ind2ptr_count_kernel<<<persistent_blocks(4), 256, 0, st>>>(index, n, size, cnt, err);
    MKG_LAUNCHED("ind2ptr_count_kernel");
  }
  if (size > 0) {
    size_t b = ws_bytes - align256(8 * (size_t)(size + 1));
    MKG_CUDA(cub::DeviceScan::InclusiveSum(temp, b, cnt + 1, ptr + 1, (int)size, st));
  }
  return MKG_OK;
}

int fact_table(const mkg_graph* g, int32_t* head, int32_t* tail, int16_t* rel, unsigned* err,
               cudaStream_t st) {
  MKG_REQUIRE(g && head && tail && rel, "fact_table: null argument");
  fact_table_kernel<<<persistent_blocks(4), 256, 0, st>>>(make_dir(g->ori), g->num_entities, g->num_facts,
                                                          head, tail, rel, err);
  MKG_LAUNCHED("fact_table_kernel");
  return MKG_OK;
}

int64_t adjacency_max_tasks(int64_t E, int64_t T) { return E + (2 * T) / kTaskSeg + 1; }

size_t adjacency_workspace_bytes(int64_t E) {
  size_t b = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, b, (int32_t*)nullptr, (int32_t*)nullptr, (int)(E + 1));
  return 2 * align256(4 * (size_t)(E + 1)) + align256(b) + 256;
}

static int build_tasks(const int32_t* ptr, int64_t E, int4* tasks, int64_t* total, void* ws, size_t ws_bytes,
                       cudaStream_t st) {
  int32_t* nt = static_cast<int32_t*>(ws);
  int32_t* offs = reinterpret_cast<int32_t*>(static_cast<char*>(ws) + align256(4 * (size_t)(E + 1)));
  void* temp = static_cast<char*>(ws) + 2 * align256(4 * (size_t)(E + 1));
  size_t tb = ws_bytes - 2 * align256(4 * (size_t)(E + 1));
  task_count_kernel<<<persistent_blocks(4), 256, 0, st>>>(ptr, E, nt);
  MKG_LAUNCHED("task_count_kernel");
  MKG_CUDA(cub::DeviceScan::ExclusiveSum(temp, tb, nt, offs, (int)(E + 1), st));
  task_fill_kernel<<<persistent_blocks(4), 256, 0, st>>>(ptr, nt, offs, E, tasks, total);
  MKG_LAUNCHED("task_fill_kernel");
  return MKG_OK;
}

int adjacency_build(const mkg_graph* g, mkg_adjacency adj, int64_t* num_tasks, void* ws, size_t ws_bytes,
                    unsigned* err, cudaStream_t st) {
  MKG_REQUIRE(g && adj.pull_ptr && adj.pull && adj.push_ptr && adj.push && adj.pull_tasks && adj.push_tasks &&
                  num_tasks, "adjacency_build: null argument");
  MKG_REQUIRE(ws && ws_bytes >= adjacency_workspace_bytes(g->num_entities), "adjacency_build: workspace too small");
  MKG_REQUIRE(2 * g->num_facts < (int64_t(1) << 31), "adjacency_build: too many facts for 32-bit offsets");
  const int64_t E = g->num_entities, T = g->num_facts, R = g->num_relations;
  const int blocks = persistent_blocks(4);
  DirCSR ori = make_dir(g->ori), inv = make_dir(g->inv);
  // pull row d: inv row d (channel rel) then ori row d (channel R + rel)
  adjacency_ptr_kernel<<<blocks, 256, 0, st>>>(inv.row_ptr, ori.row_ptr, E, adj.pull_ptr);
  MKG_LAUNCHED("adjacency_ptr_kernel");
  adjacency_fill_kernel<<<blocks, 256, 0, st>>>(inv, ori.row_ptr, E, T, 0, 0, adj.pull_ptr, adj.pull, err);
  MKG_LAUNCHED("adjacency_fill_kernel");
  adjacency_fill_kernel<<<blocks, 256, 0, st>>>(ori, inv.row_ptr, E, T, R, 1, adj.pull_ptr, adj.pull, err);
  MKG_LAUNCHED("adjacency_fill_kernel");
  // push row s: ori row s (channel rel) then inv row s (channel R + rel)
  adjacency_ptr_kernel<<<blocks, 256, 0, st>>>(ori.row_ptr, inv.row_ptr, E, adj.push_ptr);
  MKG_LAUNCHED("adjacency_ptr_kernel");
  adjacency_fill_kernel<<<blocks, 256, 0, st>>>(ori, inv.row_ptr, E, T, 0, 0, adj.push_ptr, adj.push, err);
  MKG_LAUNCHED("adjacency_fill_kernel");
  adjacency_fill_kernel<<<blocks, 256, 0, st>>>(inv, ori.row_ptr, E, T, R, 1, adj.push_ptr, adj.push, err);
  MKG_LAUNCHED("adjacency_fill_kernel");
  int rc = build_tasks(adj.pull_ptr, E, reinterpret_cast<int4*>(adj.pull_tasks), num_tasks, ws, ws_bytes, st);
  if (rc) return rc;
  return build_tasks(adj.push_ptr, E, reinterpret_cast<int4*>(adj.push_tasks), num_tasks + 1, ws, ws_bytes, st);
}

int adjacency_set_factor(const mkg_graph* g, mkg_adjacency adj, const mkg_edge_factor* f, cudaStream_t st) {
  MKG_REQUIRE(g && f, "adjacency_set_factor: null argument");
  EdgeFactor ef = make_factor(*f);
  const int64_t count = 2 * g->num_facts;
  if (adj.pull != nullptr) {  // a list passed as NULL keeps its factors
    adjacency_factor_kernel<<<persistent_blocks(8), 256, 0, st>>>(adj.pull, count, g->num_facts, ef);
    MKG_LAUNCHED("adjacency_factor_kernel");
  }
  if (adj.push != nullptr) {
    adjacency_factor_kernel<<<persistent_blocks(8), 256, 0, st>>>(adj.push, count, g->num_facts, ef);
    MKG_LAUNCHED("adjacency_factor_kernel");
  }
  return MKG_OK;
}

int records_set_factor(mkg_adj_edge* recs, int64_t count, int64_t num_facts, const mkg_edge_factor* f,
                       cudaStream_t st) {
  MKG_REQUIRE(f && count >= 0 && num_facts >= 0 && (recs || count == 0), "records_set_factor: bad argument");
  if (count == 0) return MKG_OK;
  adjacency_factor_kernel<<<grid_for(count, 256, persistent_blocks(8)), 256, 0, st>>>(recs, count, num_facts,
                                                                                     make_factor(*f));
  MKG_LAUNCHED("adjacency_factor_kernel");
  return MKG_OK;
}

// ---------------------------------------------------------------- edge-cap index
namespace {
struct CapWs {
  int32_t* flag;
  int32_t* ngrp;
  int32_t* sidx;
  int32_t* gbase;
  int2* fact_cap;
  void* temp;
  size_t temp_bytes;
};

size_t cap_scan_bytes(int64_t E) {
  size_t b = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, b, (int32_t*)nullptr, (int32_t*)nullptr, (int)(2 * E + 1));
  return b;
}

CapWs cap_ws(void* ws, int64_t E, int64_t T) {
  CapWs w;
  char* p = static_cast<char*>(ws);
  const size_t a = align256(4 * (size_t)(2 * E + 1));
  w.flag = reinterpret_cast<int32_t*>(p); p += a;
  w.ngrp = reinterpret_cast<int32_t*>(p); p += a;
  w.sidx = reinterpret_cast<int32_t*>(p); p += a;
  w.gbase = reinterpret_cast<int32_t*>(p); p += a;
  w.fact_cap = reinterpret_cast<int2*>(p); p += align256(16 * (size_t)T);
  w.temp = p;
  w.temp_bytes = cap_scan_bytes(E);
  return w;
}

// flags, group counts and their scans (slot index, first take-table row) for `cap`
int cap_scan(const mkg_graph* g, int64_t cap, const CapWs& w, int32_t* capdeg, cudaStream_t st) {
  const int64_t E = g->num_entities;
  cap_rows_kernel<<<persistent_blocks(4), 256, 0, st>>>(make_dir(g->ori), make_dir(g->inv), E, cap, w.flag, w.ngrp,
                                                        capdeg);
  MKG_LAUNCHED("cap_rows_kernel");
  size_t b = w.temp_bytes;
  MKG_CUDA(cub::DeviceScan::ExclusiveSum(w.temp, b, w.flag, w.sidx, (int)(2 * E + 1), st));
  b = w.temp_bytes;
  MKG_CUDA(cub::DeviceScan::ExclusiveSum(w.temp, b, w.ngrp, w.gbase, (int)(2 * E + 1), st));
  return MKG_OK;
}
}  // namespace

size_t cap_index_workspace_bytes(const mkg_graph* g) {
  if (!g) return 0;
  const int64_t E = g->num_entities, T = g->num_facts;
  return 4 * align256(4 * (size_t)(2 * E + 1)) + align256(16 * (size_t)T) + align256(cap_scan_bytes(E)) + 256;
}

int cap_index_sizes(const mkg_graph* g, int64_t cap, int64_t* sizes, void* ws, size_t ws_bytes, cudaStream_t st) {
  MKG_REQUIRE(g && sizes && ws, "cap_index_sizes: null argument");
  MKG_REQUIRE(cap >= 0 && cap <= MKG_DENSE_CAP_MAX, "cap_index: cap %lld outside [0, %d]", (long long)cap,
              MKG_DENSE_CAP_MAX);
  MKG_REQUIRE(2 * g->num_entities + 1 < (int64_t(1) << 31), "cap_index: too many entities");
  MKG_REQUIRE(ws_bytes >= cap_index_workspace_bytes(g), "cap_index_sizes: workspace too small");
  const CapWs w = cap_ws(ws, g->num_entities, g->num_facts);
  if (int rc = cap_scan(g, cap, w, nullptr, st)) return rc;
  cap_sizes_kernel<<<1, 1, 0, st>>>(w.sidx, w.gbase, g->num_entities, sizes);
  MKG_LAUNCHED("cap_sizes_kernel");
  return MKG_OK;
}

int cap_index_build(const mkg_graph* g, const mkg_adjacency* adj, const mkg_cap_index* ix, void* ws,
                    size_t ws_bytes, unsigned* err, cudaStream_t st) {
  MKG_REQUIRE(g && adj && ix && ws && adj->pull && adj->push, "cap_index_build: null argument");
  MKG_REQUIRE(ix->cap >= 0 && ix->cap <= MKG_DENSE_CAP_MAX, "cap_index: cap %lld outside [0, %d]",
              (long long)ix->cap, MKG_DENSE_CAP_MAX);
  MKG_REQUIRE(ix->pull_cap && ix->push_cap && ix->capped_degree &&
                  (ix->num_slots == 0 || (ix->slot_entity && ix->slot_dir && ix->slot_group)),
              "cap_index_build: null output array");
  MKG_REQUIRE(ws_bytes >= cap_index_workspace_bytes(g), "cap_index_build: workspace too small");
  const int64_t E = g->num_entities, T = g->num_facts, R = g->num_relations;
  const CapWs w = cap_ws(ws, E, T);
  if (int rc = cap_scan(g, ix->cap, w, const_cast<int32_t*>(ix->capped_degree), st)) return rc;
  const int blocks = persistent_blocks(4);
  if (ix->num_slots > 0) {
    cap_slots_kernel<<<blocks, 256, 0, st>>>(w.flag, w.sidx, w.gbase, E, ix->num_slots,
                                             const_cast<int32_t*>(ix->slot_entity), const_cast<int32_t*>(ix->slot_dir),
                                             const_cast<int32_t*>(ix->slot_group), err);
    MKG_LAUNCHED("cap_slots_kernel");
  }
  cap_fact_kernel<<<blocks, 256, 0, st>>>(make_dir(g->ori), 0, E, T, w.flag, w.gbase, w.fact_cap, err);
  MKG_LAUNCHED("cap_fact_kernel");
  cap_fact_kernel<<<blocks, 256, 0, st>>>(make_dir(g->inv), 1, E, T, w.flag, w.gbase, w.fact_cap, err);
  MKG_LAUNCHED("cap_fact_kernel");
  cap_records_kernel<<<blocks, 256, 0, st>>>(adj->pull, 2 * T, T, R, w.fact_cap,
                                             reinterpret_cast<int2*>(const_cast<int32_t*>(ix->pull_cap)));
  MKG_LAUNCHED("cap_records_kernel");
  cap_records_kernel<<<blocks, 256, 0, st>>>(adj->push, 2 * T, T, R, w.fact_cap,
                                             reinterpret_cast<int2*>(const_cast<int32_t*>(ix->push_cap)));
  MKG_LAUNCHED("cap_records_kernel");
  return MKG_OK;
}

}  // namespace mkg
