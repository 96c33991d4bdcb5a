// Rule-weight producer: the per-hop rule weights softmax(rule_logits[:, hop] / tau) of the
// hop loop (proof.py:569-571), with rule_logits from the shared parametrisation of
// SupplyGatedDRUM._shared_rule_logits (drum.py:429-438): per rule one single-layer
// bidirectional LSTM over the sequence [emb[rel]] * K + [emb[n - 1]], then a linear layer
// 2H -> n on the first K outputs.
//
// The logits depend on the query only through its target relation, so the LSTM and the
// linear layer run once per DISTINCT relation (U rows instead of B), and the softmax kernel
// gathers each query's row.  fp32 throughout (CUDA cores: the path's tolerance is fp32).
// Rows of the linear layer are (u, t, l) in that order, i.e. logits_u [U, K, L, n].
//
//   rule_lstm_fwd_kernel     block per (relation, rule, direction): K+1 sequential LSTM
//                            steps, W_hh staged in shared memory (padded rows); writes the
//                            activations for the backward and O [rows, 2H] = [h_fwd; h_bwd]
//   sgemm_kernel             the three products of the linear layer (logits = O W^T + b,
//                            grad O = G W, grad W = G^T O): 64 x 64 tiles, 4 x 4 outputs per
//                            thread, split-K into partial sums added in a fixed order
//   rule_softmax_fwd_kernel  (hop, query, rule) rows: softmax of the relation's row / tau
// Backward (no atomics; every sum in a fixed order):
//   rule_softmax_dot_kernel, rule_softmax_bwd_kernel   softmax backward summed over the
//                            queries of each relation (queries grouped by a CSR)
//   rule_colsum_kernel       grad b_lin
//   rule_lstm_bwd_kernel     backpropagation through time per (relation, rule, direction)
//   rule_lstm_wgrad_kernel   grads of W_ih, W_hh, b per (rule, direction, gate row)
//   rule_emb_grad_kernel, rule_emb_last_kernel   embedding rows: emb[rel] (first K steps),
//                            emb[n - 1] (every relation's last step)
#include <cmath>

#include "mkg_common.cuh"
#include "mkg_internal.h"

namespace mkg {
namespace {

constexpr int kMaxHidden = 112;        // 4H (H + 1) floats of W_hh must fit in shared memory
constexpr int kSoftmaxThreads = 256;   // softmax / dot: 8 warps per block
constexpr int64_t kWideRow = 2048;     // rows at least this wide get a whole block, narrower ones a warp
constexpr int kGemmBM = 64, kGemmBN = 64, kGemmBK = 16, kGemmThreads = 256;
constexpr int64_t kFillBlocks = 296;   // 2 x 148 SMs: the grid the split-K heuristic aims for

struct Dims {
  int64_t n, H, L, K, U, B;
  float tau;
};

// saved activations per (u, l, dir, t): gates i, f, g, o after activation [4H] | c [H] | h [H];
// after them O [U K L, 2H]
__device__ __forceinline__ size_t saved_at(const Dims& d, int64_t u, int64_t l, int dir, int64_t t) {
  return ((((size_t)u * d.L + l) * 2 + dir) * (d.K + 1) + t) * (size_t)(6 * d.H);
}
__host__ __device__ __forceinline__ size_t saved_o_offset(const Dims& d) {
  return (size_t)d.U * d.L * 2 * (d.K + 1) * 6 * d.H;
}
__device__ __forceinline__ size_t dpre_at(const Dims& d, int64_t u, int64_t l, int dir, int64_t t) {
  return ((((size_t)u * d.L + l) * 2 + dir) * (d.K + 1) + t) * (size_t)(4 * d.H);
}
// linear-layer row of (u, t, l) = the layout of logits_u [U, K, L, n]
__device__ __forceinline__ int64_t lin_row(const Dims& d, int64_t u, int64_t t, int64_t l) {
  return (u * d.K + t) * d.L + l;
}

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ------------------------------------------------------------------------ forward
// PyTorch's LSTM cell: gates = W_ih x + b_ih + W_hh h + b_hh, rows [i; f; g; o];
// c' = f c + i g, h' = o tanh(c').  The reverse direction walks t = K .. 0.
__global__ void rule_lstm_fwd_kernel(Dims d, const float* __restrict__ emb, const float* __restrict__ w_ih,
                                     const float* __restrict__ w_hh, const float* __restrict__ bias,
                                     const int64_t* __restrict__ rel_u, float* __restrict__ saved,
                                     unsigned* err) {
  extern __shared__ float sm[];
  const int H = (int)d.H, G = 4 * H, P = H + 1;
  float* whh = sm;           // [G][H + 1]
  float* xs = whh + G * P;   // emb[rel]
  float* xl = xs + H;        // emb[n - 1]
  float* hs = xl + H;        // hidden state
  float* gs = hs + H;        // activated gates
  const int64_t blk = blockIdx.x;
  const int dir = (int)(blk & 1);
  const int64_t l = (blk >> 1) % d.L, u = (blk >> 1) / d.L;
  const int j = threadIdx.x;
  const int64_t r = rel_u[u];
  if (r < 0 || r >= d.n) {  // uniform over the block
    if (j == 0) raise_flag(err, MKG_DEV_BAD_RULE_INDEX);
    return;
  }
  const size_t ld = (size_t)l * 2 + dir;
  const float* wh = w_hh + ld * G * H;
  for (int i = j; i < G * H; i += G) whh[(i / H) * P + (i % H)] = wh[i];
  for (int i = j; i < H; i += G) {
    xs[i] = emb[(size_t)r * H + i];
    xl[i] = emb[(size_t)(d.n - 1) * H + i];
    hs[i] = 0.0f;
  }
  __syncthreads();
  // input projections: identical for the first K steps, then the end token
  const float* wi = w_ih + (ld * G + j) * H;
  float pb = 0.0f, pl = 0.0f;
#pragma unroll 8
  for (int k = 0; k < H; ++k) {
    const float w = __ldg(wi + k);
    pb = fmaf(w, xs[k], pb);
    pl = fmaf(w, xl[k], pl);
  }
  const float b = bias[ld * G + j];
  pb += b;
  pl += b;
  const int gate = j / H;
  const float* wr = whh + j * P;
  float* o_rows = saved + saved_o_offset(d);
  float c = 0.0f;
  for (int64_t s = 0; s <= d.K; ++s) {
    const int64_t t = dir == 0 ? s : d.K - s;
    float acc = 0.0f;
    for (int k = 0; k < H; ++k) acc = fmaf(wr[k], hs[k], acc);
    const float pre = (t < d.K ? pb : pl) + acc;
    const float a = gate == 2 ? tanhf(pre) : sigmoid_f(pre);
    gs[j] = a;
    __syncthreads();  // all gates written, all reads of hs done
    float* sv = saved + saved_at(d, u, l, dir, t);
    sv[j] = a;
    if (j < H) {
      c = gs[H + j] * c + gs[j] * gs[2 * H + j];
      const float h = gs[3 * H + j] * tanhf(c);
      hs[j] = h;
      sv[G + j] = c;
      sv[G + H + j] = h;
      if (t < d.K) o_rows[(size_t)lin_row(d, u, t, l) * (2 * H) + dir * H + j] = h;
    }
    __syncthreads();
  }
}

// C (+ split z * M * N) [M, N] row-major = sum over k in split z of A(m, k) B(k, n)
// (+ bias[n] when given), with A(m, k) = A[m sam + k sak] and B(k, n) = B[k sbk + n sbn].
// Tiles are staged along whichever index is contiguous in memory, so every load coalesces.
__global__ void __launch_bounds__(kGemmThreads) sgemm_kernel(int64_t M, int64_t N, int64_t K,
                                                             const float* __restrict__ A, int64_t sam, int64_t sak,
                                                             const float* __restrict__ B, int64_t sbk, int64_t sbn,
                                                             const float* __restrict__ bias, float* __restrict__ C,
                                                             int64_t k_per_split) {
  __shared__ __align__(16) float As[kGemmBK][kGemmBM + 4];
  __shared__ __align__(16) float Bs[kGemmBK][kGemmBN + 4];
  const int tid = threadIdx.x;
  const int tm = tid / 16, tn = tid % 16;  // outputs rows tm*4 .. +3, columns tn*4 .. +3
  const int64_t m0 = (int64_t)blockIdx.y * kGemmBM, n0 = (int64_t)blockIdx.x * kGemmBN;
  const int64_t kb = (int64_t)blockIdx.z * k_per_split;
  const int64_t ke = kb + k_per_split < K ? kb + k_per_split : K;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[i][q] = 0.0f;
  for (int64_t k0 = kb; k0 < ke; k0 += kGemmBK) {
#pragma unroll
    for (int it = 0; it < kGemmBM * kGemmBK / kGemmThreads; ++it) {
      const int i = tid + it * kGemmThreads;
      int mm, kk;
      if (sak == 1) { mm = i / kGemmBK; kk = i % kGemmBK; } else { kk = i / kGemmBM; mm = i % kGemmBM; }
      const int64_t m = m0 + mm, k = k0 + kk;
      As[kk][mm] = (m < M && k < ke) ? A[m * sam + k * sak] : 0.0f;
    }
#pragma unroll
    for (int it = 0; it < kGemmBN * kGemmBK / kGemmThreads; ++it) {
      const int i = tid + it * kGemmThreads;
      int nn, kk;
      if (sbn == 1) { kk = i / kGemmBN; nn = i % kGemmBN; } else { nn = i / kGemmBK; kk = i % kGemmBK; }
      const int64_t nc = n0 + nn, k = k0 + kk;
      Bs[kk][nn] = (nc < N && k < ke) ? B[k * sbk + nc * sbn] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kGemmBK; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&As[kk][tm * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tn * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[i][q] = fmaf(av[i], bv[q], acc[i][q]);
    }
    __syncthreads();
  }
  float* out = C + (size_t)blockIdx.z * M * N;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + tm * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int64_t nc = n0 + tn * 4 + q;
      if (nc < N) out[(size_t)m * N + nc] = acc[i][q] + (bias ? bias[nc] : 0.0f);
    }
  }
}

// out[i] = sum over splits s (in order) of part[s * count + i]
__global__ void split_reduce_kernel(int64_t count, int64_t splits, const float* __restrict__ part,
                                    float* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int64_t p = 0; p < splits; ++p) s += part[(size_t)p * count + i];
    out[i] = s;
  }
}

// Reductions over the WPR warps of one row (sums in warp order: the same result every run).
template <int WPR>
__device__ __forceinline__ float row_max(float v, float* red) {
  v = warp_max(v);
  if (WPR == 1) return v;
  if (threadIdx.x % kWarp == 0) red[threadIdx.x / kWarp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < WPR; ++i) r = fmaxf(r, red[i]);
  __syncthreads();
  return r;
}
template <int WPR>
__device__ __forceinline__ float row_sum(float v, float* red) {
  v = warp_sum(v);
  if (WPR == 1) return v;
  if (threadIdx.x % kWarp == 0) red[threadIdx.x / kWarp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < WPR; ++i) r += red[i];
  __syncthreads();
  return r;
}

// w_hops[t, b, l, :] = softmax(logits_u[query_u[b], t, l, :] / tau); WPR warps per row
// (1: eight rows per block; 8: one row per block, every exit below is uniform over the block)
template <int WPR>
__global__ void __launch_bounds__(kSoftmaxThreads) rule_softmax_fwd_kernel(
    Dims d, const float* __restrict__ logits, const int64_t* __restrict__ query_u, float* __restrict__ w_hops,
    unsigned* err) {
  __shared__ float red[kSoftmaxThreads / kWarp];
  constexpr int kStride = kWarp * WPR;
  const int64_t row = (int64_t)blockIdx.x * (kSoftmaxThreads / kStride) + threadIdx.x / kStride;
  const int lane = threadIdx.x % kStride;
  if (row >= d.K * d.B * d.L) return;
  const int64_t l = row % d.L, b = (row / d.L) % d.B, t = row / (d.L * d.B);
  const int64_t u = query_u[b];
  if (u < 0 || u >= d.U) {
    if (lane == 0) raise_flag(err, MKG_DEV_BAD_RULE_INDEX);
    return;
  }
  const float* x = logits + (size_t)lin_row(d, u, t, l) * d.n;
  float* y = w_hops + (size_t)row * d.n;
  float m = -INFINITY;
  for (int64_t c = lane; c < d.n; c += kStride) m = fmaxf(m, x[c] / d.tau);
  m = row_max<WPR>(m, red);
  float s = 0.0f;
  for (int64_t c = lane; c < d.n; c += kStride) s += expf(x[c] / d.tau - m);
  s = row_sum<WPR>(s, red);
  for (int64_t c = lane; c < d.n; c += kStride) y[c] = expf(x[c] / d.tau - m) / s;
}

// ----------------------------------------------------------------------- backward
// dot[row] = sum_c w[row, c] g[row, c]
template <int WPR>
__global__ void __launch_bounds__(kSoftmaxThreads) rule_softmax_dot_kernel(Dims d, const float* __restrict__ w,
                                                                           const float* __restrict__ g,
                                                                           float* __restrict__ dot) {
  __shared__ float red[kSoftmaxThreads / kWarp];
  constexpr int kStride = kWarp * WPR;
  const int64_t row = (int64_t)blockIdx.x * (kSoftmaxThreads / kStride) + threadIdx.x / kStride;
  const int lane = threadIdx.x % kStride;
  if (row >= d.K * d.B * d.L) return;
  const float* wr = w + (size_t)row * d.n;
  const float* gr = g + (size_t)row * d.n;
  float s = 0.0f;
  for (int64_t c = lane; c < d.n; c += kStride) s = fmaf(wr[c], gr[c], s);
  s = row_sum<WPR>(s, red);
  if (lane == 0) dot[row] = s;
}

// grad_logits_u[u, t, l, c] = sum over the queries b of u (CSR order) of
// w[t, b, l, c] (g[t, b, l, c] - dot[t, b, l]) / tau
__global__ void rule_softmax_bwd_kernel(Dims d, const float* __restrict__ w, const float* __restrict__ g,
                                        const float* __restrict__ dot, const int64_t* __restrict__ qptr,
                                        const int64_t* __restrict__ qperm, float* __restrict__ grad_logits,
                                        unsigned* err) {
  const int64_t c = (int64_t)blockIdx.y * blockDim.x + threadIdx.x;
  const int64_t urow = blockIdx.x;  // (u, t, l)
  if (c >= d.n) return;
  const int64_t l = urow % d.L, t = (urow / d.L) % d.K, u = urow / (d.L * d.K);
  const int64_t q0 = qptr[u], q1 = qptr[u + 1];
  float acc = 0.0f;
  for (int64_t q = q0; q < q1; ++q) {
    const int64_t b = qperm[q];
    if (b < 0 || b >= d.B) {
      raise_flag(err, MKG_DEV_BAD_RULE_INDEX);
      continue;
    }
    const int64_t row = (t * d.B + b) * d.L + l;
    const size_t at = (size_t)row * d.n + c;
    acc += w[at] * (g[at] - dot[row]);
  }
  grad_logits[(size_t)urow * d.n + c] = acc / d.tau;
}

// grad b_lin[c] = sum over rows (in order) of gl[row, c]
__global__ void rule_colsum_kernel(int64_t rows, int64_t n, const float* __restrict__ gl, float* __restrict__ out) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  float s = 0.0f;
  for (int64_t r = 0; r < rows; ++r) s += gl[(size_t)r * n + c];
  out[c] = s;
}

// Backpropagation through time for one (u, l, dir).  Writes the pre-activation gate
// gradients (for the weight gradients) and the per-block input gradients:
// part[(u, l, dir), 0, :] = sum over the first K steps (emb[rel]), part[.., 1, :] = the last step.
// The hidden / input gradient products W^T dpre are split over the four gate blocks (one
// per group of H threads) and added in gate order.
__global__ void rule_lstm_bwd_kernel(Dims d, const float* __restrict__ w_ih, const float* __restrict__ w_hh,
                                     const float* __restrict__ saved, const float* __restrict__ grad_o,
                                     float* __restrict__ dpre_ws, float* __restrict__ part) {
  extern __shared__ float sm[];
  const int H = (int)d.H, G = 4 * H;
  float* dp = sm;           // [G]
  float* ph = dp + G;       // [4][H] partial W_hh^T dpre
  float* px = ph + G;       // [4][H] partial W_ih^T dpre
  const int64_t blk = blockIdx.x;
  const int dir = (int)(blk & 1);
  const int64_t l = (blk >> 1) % d.L, u = (blk >> 1) / d.L;
  const int tid = threadIdx.x;
  const int q = tid / H, jq = tid % H;  // gate block q, column jq
  const size_t ld = (size_t)l * 2 + dir;
  const float* wi = w_ih + ld * G * H;
  const float* wh = w_hh + ld * G * H;
  float dh_carry = 0.0f, dc_next = 0.0f, dx_base = 0.0f, dx_last = 0.0f;
  for (int64_t s = d.K; s >= 0; --s) {
    const int64_t t = dir == 0 ? s : d.K - s;
    if (tid < H) {
      const int j = tid;
      const float* sv = saved + saved_at(d, u, l, dir, t);
      const float gi = sv[j], gf = sv[H + j], gg = sv[2 * H + j], go = sv[3 * H + j], c = sv[G + j];
      float c_prev = 0.0f;
      if (s > 0) c_prev = saved[saved_at(d, u, l, dir, dir == 0 ? t - 1 : t + 1) + G + j];
      float dh = dh_carry;
      if (t < d.K) dh += grad_o[(size_t)lin_row(d, u, t, l) * (2 * H) + dir * H + j];
      const float tc = tanhf(c);
      const float d_o = dh * tc;
      const float dc = dc_next + dh * go * (1.0f - tc * tc);
      const float d_i = dc * gg, d_f = dc * c_prev, d_g = dc * gi;
      dc_next = dc * gf;
      dp[j] = d_i * gi * (1.0f - gi);
      dp[H + j] = d_f * gf * (1.0f - gf);
      dp[2 * H + j] = d_g * (1.0f - gg * gg);
      dp[3 * H + j] = d_o * go * (1.0f - go);
    }
    __syncthreads();
    dpre_ws[dpre_at(d, u, l, dir, t) + tid] = dp[tid];
    {
      float ah = 0.0f, ax = 0.0f;
      const int r0 = q * H;
#pragma unroll 8
      for (int r = 0; r < H; ++r) {
        const float g = dp[r0 + r];
        ah = fmaf(wh[(size_t)(r0 + r) * H + jq], g, ah);
        ax = fmaf(wi[(size_t)(r0 + r) * H + jq], g, ax);
      }
      ph[q * H + jq] = ah;
      px[q * H + jq] = ax;
    }
    __syncthreads();
    if (tid < H) {
      dh_carry = ((ph[tid] + ph[H + tid]) + ph[2 * H + tid]) + ph[3 * H + tid];
      const float ax = ((px[tid] + px[H + tid]) + px[2 * H + tid]) + px[3 * H + tid];
      if (t < d.K) dx_base += ax; else dx_last += ax;
    }
    __syncthreads();
  }
  if (tid < H) {
    float* pp = part + ((((size_t)u * d.L + l) * 2 + dir) * 2) * H;
    pp[tid] = dx_base;
    pp[H + tid] = dx_last;
  }
}

// grad W_ih / W_hh rows and bias of (l, dir, gate row j): sums over u, then t, of
// dpre[j] * x_t[k] and dpre[j] * h_{t-1}[k] (h of the previous step in walk order, 0 first)
__global__ void rule_lstm_wgrad_kernel(Dims d, const float* __restrict__ emb, const int64_t* __restrict__ rel_u,
                                       const float* __restrict__ saved, const float* __restrict__ dpre_ws,
                                       float* __restrict__ grad_w_ih, float* __restrict__ grad_w_hh,
                                       float* __restrict__ grad_bias) {
  const int H = (int)d.H, G = 4 * H;
  const int64_t blk = blockIdx.x;
  const int j = (int)(blk % G);
  const int64_t ld = blk / G;  // l * 2 + dir
  const int dir = (int)(ld & 1);
  const int64_t l = ld >> 1;
  const int k = threadIdx.x;
  float aih = 0.0f, ahh = 0.0f, ab = 0.0f;
  const float xl = emb[(size_t)(d.n - 1) * H + k];
#pragma unroll 2
  for (int64_t u = 0; u < d.U; ++u) {
    const int64_t r = rel_u[u];
    if (r < 0 || r >= d.n) continue;  // flagged by the forward
    const float xb = emb[(size_t)r * H + k];
    for (int64_t t = 0; t <= d.K; ++t) {
      const float g = dpre_ws[dpre_at(d, u, l, dir, t) + j];
      const bool first = dir == 0 ? t == 0 : t == d.K;
      const float hp = first ? 0.0f : saved[saved_at(d, u, l, dir, dir == 0 ? t - 1 : t + 1) + 5 * H + k];
      aih = fmaf(g, t < d.K ? xb : xl, aih);
      ahh = fmaf(g, hp, ahh);
      ab += g;
    }
  }
  const size_t at = ((size_t)ld * G + j) * H + k;
  grad_w_ih[at] = aih;
  grad_w_hh[at] = ahh;
  if (k == 0) grad_bias[(size_t)ld * G + j] = ab;
}

// Row rel_u[u] of the embedding gradient (relations other than n - 1): the sum of its rules'
// and directions' first-K input gradients.  grad_emb is zeroed before.
__global__ void rule_emb_grad_kernel(Dims d, const int64_t* __restrict__ rel_u, const float* __restrict__ part,
                                     float* __restrict__ grad_emb) {
  const int H = (int)d.H;
  const int k = threadIdx.x;
  const int64_t u = blockIdx.x;
  const size_t per_u = (size_t)d.L * 2 * 2 * H;
  const int64_t r = rel_u[u];
  if (r < 0 || r >= d.n - 1) return;
  float s = 0.0f;
  for (int64_t q = 0; q < d.L * 2; ++q) s += part[u * per_u + (size_t)q * 2 * H + k];
  grad_emb[(size_t)r * H + k] = s;
}

// Row n - 1 (the end token of every sequence): block k sums, over every (u, l, dir), the
// last-step input gradient, plus the first-K gradients of a relation equal to n - 1.
__global__ void __launch_bounds__(256) rule_emb_last_kernel(Dims d, const int64_t* __restrict__ rel_u,
                                                            const float* __restrict__ part,
                                                            float* __restrict__ grad_emb) {
  __shared__ float red[256];
  const int H = (int)d.H;
  const int k = blockIdx.x;
  const int64_t items = d.U * d.L * 2;
  float s = 0.0f;
  for (int64_t v = threadIdx.x; v < items; v += blockDim.x) {
    const float* pp = part + (size_t)v * 2 * H;
    s += pp[H + k];
    if (rel_u[v / (d.L * 2)] == d.n - 1) s += pp[k];
  }
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if ((int)threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) grad_emb[(size_t)(d.n - 1) * H + k] = red[0];
}

int check_params(const mkg_rule_params* p, Dims* d) {
  MKG_REQUIRE(p != nullptr, "rule producer: null params");
  MKG_REQUIRE(p->n >= 1 && p->L >= 1 && p->K >= 1 && p->U >= 1 && p->B >= 1,
              "rule producer: sizes must be positive (n=%lld L=%lld K=%lld U=%lld B=%lld)", (long long)p->n,
              (long long)p->L, (long long)p->K, (long long)p->U, (long long)p->B);
  MKG_REQUIRE(p->H >= 1 && p->H <= kMaxHidden, "rule producer: hidden size %lld outside [1, %d]", (long long)p->H,
              kMaxHidden);
  MKG_REQUIRE(p->tau > 0.0f && std::isfinite(p->tau), "rule producer: tau must be positive");
  MKG_REQUIRE(p->U * p->L * 2 * 4 * kMaxHidden < (int64_t(1) << 31) && p->K * p->B * p->L < (int64_t(1) << 33) &&
                  p->U * p->K * p->L < 65535LL * kGemmBM,
              "rule producer: too many rows");
  MKG_REQUIRE(p->n <= 65535LL * kGemmBM, "rule producer: more than %lld channels", 65535LL * kGemmBM);
  d->n = p->n; d->H = p->H; d->L = p->L; d->K = p->K; d->U = p->U; d->B = p->B; d->tau = p->tau;
  return MKG_OK;
}

// Split-K of an [M, N] product with reduction length K: enough blocks to fill the GPU (a pure
// function of the sizes, so it also sizes the workspace).
int64_t gemm_k_per_split(int64_t M, int64_t N, int64_t K) {
  const int64_t tiles = ((M + kGemmBM - 1) / kGemmBM) * ((N + kGemmBN - 1) / kGemmBN);
  const int64_t steps = (K + kGemmBK - 1) / kGemmBK;
  int64_t splits = (kFillBlocks + tiles - 1) / tiles;
  splits = splits < 1 ? 1 : (splits > steps ? steps : splits);
  if (splits > 65535) splits = 65535;
  if (splits < 1) splits = 1;
  return ((steps + splits - 1) / splits) * kGemmBK;
}
int64_t gemm_splits(int64_t M, int64_t N, int64_t K) {
  const int64_t per = gemm_k_per_split(M, N, K);
  return K <= 0 || per <= 0 ? 1 : (K + per - 1) / per;
}

// C [M, N] = A B (+ bias); with more than one split the partial products go to `part`
// (splits * M * N floats) and are added in split order into C.
int sgemm(int64_t M, int64_t N, int64_t K, const float* A, int64_t sam, int64_t sak, const float* B, int64_t sbk,
          int64_t sbn, const float* bias, float* C, float* part, cudaStream_t st) {
  const int64_t per = gemm_k_per_split(M, N, K), splits = gemm_splits(M, N, K);
  dim3 grid((unsigned)((N + kGemmBN - 1) / kGemmBN), (unsigned)((M + kGemmBM - 1) / kGemmBM), (unsigned)splits);
  if (splits == 1) {
    sgemm_kernel<<<grid, kGemmThreads, 0, st>>>(M, N, K, A, sam, sak, B, sbk, sbn, bias, C, per);
    MKG_LAUNCHED("sgemm_kernel");
    return MKG_OK;
  }
  if (bias != nullptr || part == nullptr) { set_error("sgemm: split-K needs a partial buffer and no bias"); return MKG_ERR_ARG; }
  sgemm_kernel<<<grid, kGemmThreads, 0, st>>>(M, N, K, A, sam, sak, B, sbk, sbn, nullptr, part, per);
  MKG_LAUNCHED("sgemm_kernel");
  split_reduce_kernel<<<grid_for(M * N, 256, persistent_blocks(4)), 256, 0, st>>>(M * N, splits, part, C);
  MKG_LAUNCHED("split_reduce_kernel");
  return MKG_OK;
}

}  // namespace

size_t rule_saved_bytes(const mkg_rule_params* p) {
  if (!p || p->U < 1 || p->L < 1 || p->K < 1 || p->H < 1) return 0;
  const size_t steps = (size_t)p->U * p->L * 2 * (p->K + 1) * 6 * p->H;
  const size_t o = (size_t)p->U * p->K * p->L * 2 * p->H;
  return (steps + o) * sizeof(float);
}

size_t rule_backward_workspace_bytes(const mkg_rule_params* p) {
  if (!p || p->U < 1 || p->L < 1 || p->K < 1 || p->H < 1 || p->n < 1) return 0;
  const int64_t rows = p->U * p->K * p->L, H2 = 2 * p->H;
  const size_t go = (size_t)rows * H2;
  const size_t dp = (size_t)p->U * p->L * 2 * (p->K + 1) * 4 * p->H;
  const size_t pt = (size_t)p->U * p->L * 2 * 2 * p->H;
  const int64_t so = gemm_splits(rows, H2, p->n), sw = gemm_splits(p->n, H2, rows);
  const size_t part_o = so > 1 ? (size_t)so * rows * H2 : 0;
  const size_t part_w = sw > 1 ? (size_t)sw * p->n * H2 : 0;
  return (go + dp + pt + (part_o > part_w ? part_o : part_w)) * sizeof(float);
}

size_t rule_softmax_workspace_bytes(const mkg_rule_params* p) {
  if (!p || p->K < 1 || p->B < 1 || p->L < 1) return 0;
  return (size_t)p->K * p->B * p->L * sizeof(float);
}

int rule_logits_forward(const mkg_rule_params* p, const float* emb, const float* w_ih, const float* w_hh,
                        const float* bias, const float* w_lin, const float* b_lin, const int64_t* rel_u,
                        float* logits_u, void* saved, size_t saved_bytes, unsigned* err, cudaStream_t st) {
  Dims d;
  if (int rc = check_params(p, &d)) return rc;
  MKG_REQUIRE(emb && w_ih && w_hh && bias && w_lin && b_lin && rel_u && logits_u && saved,
              "rule_logits_forward: null argument");
  if (saved_bytes < rule_saved_bytes(p)) {
    set_error("rule_logits_forward: saved buffer %zu < %zu bytes", saved_bytes, rule_saved_bytes(p));
    return MKG_ERR_CAPACITY;
  }
  const int H = (int)d.H, G = 4 * H;
  float* sv = static_cast<float*>(saved);
  const size_t sm_lstm = ((size_t)G * (H + 1) + 3 * H + G) * sizeof(float);
  MKG_CUDA(cudaFuncSetAttribute(rule_lstm_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_lstm));
  rule_lstm_fwd_kernel<<<(unsigned)(d.U * d.L * 2), G, sm_lstm, st>>>(d, emb, w_ih, w_hh, bias, rel_u, sv, err);
  MKG_LAUNCHED("rule_lstm_fwd_kernel");
  // logits [rows, n] = O [rows, 2H] W_lin^T + b_lin; the reduction (2H) is short: one split
  const int64_t rows = d.U * d.K * d.L;
  const float* o = sv + saved_o_offset(d);
  dim3 grid((unsigned)((d.n + kGemmBN - 1) / kGemmBN), (unsigned)((rows + kGemmBM - 1) / kGemmBM), 1);
  sgemm_kernel<<<grid, kGemmThreads, 0, st>>>(rows, d.n, 2 * H, o, 2 * H, 1, w_lin, 1, 2 * H, b_lin, logits_u,
                                              2 * H);
  MKG_LAUNCHED("sgemm_kernel");
  return MKG_OK;
}

int rule_softmax_forward(const mkg_rule_params* p, const float* logits_u, const int64_t* query_u, float* w_hops,
                         unsigned* err, cudaStream_t st) {
  Dims d;
  if (int rc = check_params(p, &d)) return rc;
  MKG_REQUIRE(logits_u && query_u && w_hops, "rule_softmax_forward: null argument");
  const int64_t rows = d.K * d.B * d.L;
  constexpr int64_t kNarrowRows = kSoftmaxThreads / kWarp;
  if (d.n >= kWideRow)
    rule_softmax_fwd_kernel<8><<<(unsigned)rows, kSoftmaxThreads, 0, st>>>(d, logits_u, query_u, w_hops, err);
  else
    rule_softmax_fwd_kernel<1><<<(unsigned)((rows + kNarrowRows - 1) / kNarrowRows), kSoftmaxThreads, 0, st>>>(
        d, logits_u, query_u, w_hops, err);
  MKG_LAUNCHED("rule_softmax_fwd_kernel");
  return MKG_OK;
}

int rule_softmax_backward(const mkg_rule_params* p, const float* w_hops, const float* grad_w_hops,
                          const int64_t* query_ptr, const int64_t* query_perm, float* grad_logits_u, void* ws,
                          size_t ws_bytes, unsigned* err, cudaStream_t st) {
  Dims d;
  if (int rc = check_params(p, &d)) return rc;
  MKG_REQUIRE(w_hops && grad_w_hops && query_ptr && query_perm && grad_logits_u && ws,
              "rule_softmax_backward: null argument");
  if (ws_bytes < rule_softmax_workspace_bytes(p)) {
    set_error("rule_softmax_backward: workspace %zu < %zu bytes", ws_bytes, rule_softmax_workspace_bytes(p));
    return MKG_ERR_CAPACITY;
  }
  float* dot = static_cast<float*>(ws);
  const int64_t rows = d.K * d.B * d.L;
  constexpr int64_t kNarrowRows = kSoftmaxThreads / kWarp;
  if (d.n >= kWideRow)
    rule_softmax_dot_kernel<8><<<(unsigned)rows, kSoftmaxThreads, 0, st>>>(d, w_hops, grad_w_hops, dot);
  else
    rule_softmax_dot_kernel<1><<<(unsigned)((rows + kNarrowRows - 1) / kNarrowRows), kSoftmaxThreads, 0, st>>>(
        d, w_hops, grad_w_hops, dot);
  MKG_LAUNCHED("rule_softmax_dot_kernel");
  dim3 grid((unsigned)(d.U * d.K * d.L), (unsigned)((d.n + 255) / 256));
  rule_softmax_bwd_kernel<<<grid, 256, 0, st>>>(d, w_hops, grad_w_hops, dot, query_ptr, query_perm, grad_logits_u,
                                               err);
  MKG_LAUNCHED("rule_softmax_bwd_kernel");
  return MKG_OK;
}

int rule_logits_backward(const mkg_rule_params* p, const float* emb, const float* w_ih, const float* w_hh,
                         const float* w_lin, const int64_t* rel_u, const void* saved, size_t saved_bytes,
                         const float* grad_logits_u, float* grad_emb, float* grad_w_ih, float* grad_w_hh,
                         float* grad_bias, float* grad_w_lin, float* grad_b_lin, void* ws, size_t ws_bytes,
                         unsigned* err, cudaStream_t st) {
  (void)err;
  Dims d;
  if (int rc = check_params(p, &d)) return rc;
  MKG_REQUIRE(emb && w_ih && w_hh && w_lin && rel_u && saved && grad_logits_u && grad_emb && grad_w_ih &&
                  grad_w_hh && grad_bias && grad_w_lin && grad_b_lin && ws,
              "rule_logits_backward: null argument");
  if (saved_bytes < rule_saved_bytes(p)) {
    set_error("rule_logits_backward: saved buffer %zu < %zu bytes", saved_bytes, rule_saved_bytes(p));
    return MKG_ERR_CAPACITY;
  }
  if (ws_bytes < rule_backward_workspace_bytes(p)) {
    set_error("rule_logits_backward: workspace %zu < %zu bytes", ws_bytes, rule_backward_workspace_bytes(p));
    return MKG_ERR_CAPACITY;
  }
  const int H = (int)d.H, G = 4 * H, H2 = 2 * H;
  const int64_t rows = d.U * d.K * d.L;
  const float* sv = static_cast<const float*>(saved);
  const float* o = sv + saved_o_offset(d);
  float* grad_o = static_cast<float*>(ws);
  float* dpre = grad_o + (size_t)rows * H2;
  float* part = dpre + (size_t)d.U * d.L * 2 * (d.K + 1) * G;
  float* gemm_part = part + (size_t)d.U * d.L * 2 * 2 * H;
  // grad W_lin [n, 2H] = G^T O (reduction over rows); grad b_lin = column sums of G
  if (int rc = sgemm(d.n, H2, rows, grad_logits_u, 1, d.n, o, H2, 1, nullptr, grad_w_lin, gemm_part, st)) return rc;
  rule_colsum_kernel<<<(unsigned)((d.n + 255) / 256), 256, 0, st>>>(rows, d.n, grad_logits_u, grad_b_lin);
  MKG_LAUNCHED("rule_colsum_kernel");
  // grad O [rows, 2H] = G W_lin (reduction over the n channels)
  if (int rc = sgemm(rows, H2, d.n, grad_logits_u, d.n, 1, w_lin, H2, 1, nullptr, grad_o, gemm_part, st)) return rc;
  rule_lstm_bwd_kernel<<<(unsigned)(d.U * d.L * 2), G, 3 * G * sizeof(float), st>>>(d, w_ih, w_hh, sv, grad_o,
                                                                                    dpre, part);
  MKG_LAUNCHED("rule_lstm_bwd_kernel");
  rule_lstm_wgrad_kernel<<<(unsigned)(d.L * 2 * G), H, 0, st>>>(d, emb, rel_u, sv, dpre, grad_w_ih, grad_w_hh,
                                                                grad_bias);
  MKG_LAUNCHED("rule_lstm_wgrad_kernel");
  MKG_CUDA(cudaMemsetAsync(grad_emb, 0, (size_t)d.n * H * sizeof(float), st));
  rule_emb_grad_kernel<<<(unsigned)d.U, H, 0, st>>>(d, rel_u, part, grad_emb);
  MKG_LAUNCHED("rule_emb_grad_kernel");
  rule_emb_last_kernel<<<(unsigned)H, 256, 0, st>>>(d, rel_u, part, grad_emb);
  MKG_LAUNCHED("rule_emb_last_kernel");
  return MKG_OK;
}

}  // namespace mkg
