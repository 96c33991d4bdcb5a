// Shared device helpers for the minikg_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstdarg>
#include <cstdio>

#include "minikg_b200.h"

namespace mkg {

constexpr int kWarp = 32;
constexpr int kNumBuckets = 256;  // edge-cap histogram (256 weight buckets)

// ---------------------------------------------------------------- host errors
void set_error(const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);

#define MKG_CUDA(call)                                   \
  do {                                                   \
    cudaError_t _e = (call);                             \
    if (_e != cudaSuccess) return ::mkg::cuda_fail(_e, #call); \
  } while (0)

#define MKG_LAUNCHED(what)                                \
  do {                                                    \
    cudaError_t _e = cudaGetLastError();                  \
    if (_e != cudaSuccess) return ::mkg::cuda_fail(_e, what); \
  } while (0)

#define MKG_REQUIRE(cond, ...)                            \
  do {                                                    \
    if (!(cond)) { ::mkg::set_error(__VA_ARGS__); return MKG_ERR_ARG; } \
  } while (0)

inline int grid_for(int64_t work, int per_block, int max_blocks) {
  int64_t g = (work + per_block - 1) / per_block;
  if (g < 1) g = 1;
  if (g > max_blocks) g = max_blocks;
  return static_cast<int>(g);
}

// Persistent-style grid: a few resident blocks per SM (148 SMs on B200).
int num_sms();
inline int persistent_blocks(int per_sm) { return num_sms() * per_sm; }

// ---------------------------------------------------------------- device side
__device__ __forceinline__ void raise_flag(unsigned* err, unsigned bit) {
  if (err) atomicOr(err, bit);
}

// Division of a non-negative key (below 2^52) by a fixed divisor through its fp64 reciprocal:
// the product's truncation is off by at most one, which one remainder test corrects.  A
// 64-bit integer division is a long emulated sequence on the GPU; this is a multiply, two
// conversions and a compare.
struct FastDiv {
  int64_t d;
  double inv;
  __host__ __device__ static FastDiv of(int64_t d) { return FastDiv{d, d > 0 ? 1.0 / (double)d : 0.0}; }
  __device__ __forceinline__ int64_t div(int64_t n) const {
    int64_t q = static_cast<int64_t>(static_cast<double>(n) * inv);
    const int64_t r = n - q * d;
    if (r < 0) --q;
    else if (r >= d) ++q;
    return q;
  }
};

// Order-preserving 32-bit key of a float (larger float -> larger key; -0 < +0).
__device__ __forceinline__ uint32_t float_order_key(float v) {
  uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float float_from_order_key(uint32_t k) {
  uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(b);
}
// (value, rank) packed so that the larger value wins and, on equal values, the
// smaller rank wins.  0 is "empty": every real pair packs to a nonzero word
// because ranks stay below 0xFFFFFFFF.
__device__ __forceinline__ unsigned long long pack_value_rank(float v, uint32_t rank) {
  return (static_cast<unsigned long long>(float_order_key(v)) << 32) |
         static_cast<unsigned long long>(0xFFFFFFFFu - rank);
}
__device__ __forceinline__ float packed_value(unsigned long long p) {
  return float_from_order_key(static_cast<uint32_t>(p >> 32));
}
__device__ __forceinline__ uint32_t packed_rank(unsigned long long p) {
  return 0xFFFFFFFFu - static_cast<uint32_t>(p & 0xFFFFFFFFull);
}

// Weight bucket of the edge cap: min(max(int(w * 255), 0), 255) with C truncation.
__device__ __forceinline__ int weight_bucket(float w) {
  float y = w * 255.0f;
  y = fminf(fmaxf(y, -1.0f), 256.0f);  // NaN-free range before the integer cast
  int b = static_cast<int>(y);
  return min(max(b, 0), kNumBuckets - 1);
}

// Edge factor m = bool(mask[e]) * score(e).
struct EdgeFactor {
  const void* mask;      // nullptr: every fact on
  int mask_kind;         // MKG_MASK_NONE / MKG_MASK_U8 / MKG_MASK_F32
  int64_t mask_numel;    // 1: broadcast to all facts
  const float* weight;   // nullptr: no score factor
  int is_score;          // 1: score = weight[e]; 0: score = sigmoid(weight[e] * scale)
  float scale;

  __device__ __forceinline__ float operator()(int64_t eid) const {
    float m = 1.0f;
    if (mask_kind != MKG_MASK_NONE && mask != nullptr) {
      int64_t idx = mask_numel == 1 ? 0 : eid;
      bool on = mask_kind == MKG_MASK_U8 ? (static_cast<const uint8_t*>(mask)[idx] != 0)
                                         : (static_cast<const float*>(mask)[idx] != 0.0f);
      m = on ? 1.0f : 0.0f;
    }
    if (weight != nullptr) {
      float ew = weight[eid];
      float s;
      if (is_score) {
        s = ew;
      } else {
        // float32 product as in the reference, sigmoid rounded from double
        float z = -ew * scale;
        s = static_cast<float>(1.0 / (1.0 + exp(static_cast<double>(z))));
      }
      m = m * s;
    }
    return m;
  }
};

inline EdgeFactor make_factor(const mkg_edge_factor& f) {
  EdgeFactor e;
  e.mask = f.mask;
  e.mask_kind = f.mask == nullptr ? MKG_MASK_NONE : f.mask_kind;
  e.mask_numel = f.mask_numel;
  e.weight = f.edge_weight_numel > 0 ? f.edge_weight : nullptr;
  e.is_score = f.is_score;
  e.scale = f.scale;
  return e;
}

struct DirCSR {
  const int32_t* row_ptr;
  const int32_t* col;
  const int16_t* rel;
  const int32_t* order;
  const int32_t* group_ptr;
  const int16_t* group_rel;
  const int32_t* group_start;
  const int32_t* group_count;
};

inline DirCSR make_dir(const mkg_csr_dir& d) {
  return DirCSR{d.row_ptr, d.col_ind, d.r_ind, d.order, d.row_group_ptr, d.group_rel,
                d.group_edge_start, d.group_edge_count};
}

// ---------------------------------------------------------------- TMA bulk copies
// One-dimensional bulk copies global -> shared completed on an mbarrier (this CTA only).
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// bytes must be a multiple of 16 and both addresses 16-byte aligned
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(done) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return done != 0;
}
// Bounded wait on one phase of an mbarrier; false when it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t max_polls) {
  for (uint32_t i = 0; i < max_polls; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ int warp_inclusive_scan(int x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  return x;
}
__device__ __forceinline__ long long warp_inclusive_scan_ll(long long x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    long long y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ double warp_sum_f64(double x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

}  // namespace mkg
