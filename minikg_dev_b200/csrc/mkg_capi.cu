// C ABI of the library: argument checks, error reporting and dispatch to the kernels.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "mkg_common.cuh"
#include "mkg_internal.h"

#define MKG_API extern "C" __attribute__((visibility("default")))

namespace mkg {

static thread_local char g_last_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int cuda_fail(cudaError_t e, const char* what) {
  set_error("CUDA error %d (%s) in %s", static_cast<int>(e), cudaGetErrorString(e), what);
  return MKG_ERR_CUDA;
}

int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

}  // namespace mkg

using mkg::set_error;

static cudaStream_t S(mkg_stream s) { return reinterpret_cast<cudaStream_t>(s); }

MKG_API const char* mkg_last_error(void) { return mkg::g_last_error; }
MKG_API int mkg_abi_version(void) { return 6; }

MKG_API size_t mkg_csr_build_workspace_bytes(int64_t T, int64_t E, int64_t R) {
  return mkg::csr_build_workspace_bytes(T, E, R);
}
MKG_API int mkg_csr_build(const int32_t* head, const int32_t* rel, const int32_t* tail, int64_t T, int64_t E,
                          int64_t R, mkg_csr_dir_out ori, mkg_csr_dir_out inv, int64_t* num_groups, void* ws,
                          size_t ws_bytes, unsigned* err, mkg_stream st) {
  if (!head || !rel || !tail || !num_groups) { set_error("csr_build: null argument"); return MKG_ERR_ARG; }
  return mkg::csr_build(head, rel, tail, T, E, R, ori, inv, num_groups, ws, ws_bytes, err, S(st));
}

MKG_API size_t mkg_ind2ptr_workspace_bytes(int64_t size) { return mkg::ind2ptr_workspace_bytes(size); }
MKG_API int mkg_ind2ptr(const int64_t* index, int64_t n, int64_t size, int64_t* ptr, void* ws, size_t ws_bytes,
                        unsigned* err, mkg_stream st) {
  if ((!index && n > 0) || !ptr) { set_error("ind2ptr: null argument"); return MKG_ERR_ARG; }
  return mkg::ind2ptr(index, n, size, ptr, ws, ws_bytes, err, S(st));
}

MKG_API int mkg_fact_table(const mkg_graph* g, int32_t* head, int32_t* tail, int16_t* rel, unsigned* err,
                           mkg_stream st) {
  return mkg::fact_table(g, head, tail, rel, err, S(st));
}

MKG_API int64_t mkg_adjacency_max_tasks(int64_t E, int64_t T) { return mkg::adjacency_max_tasks(E, T); }
MKG_API size_t mkg_adjacency_workspace_bytes(int64_t E) { return mkg::adjacency_workspace_bytes(E); }
MKG_API int mkg_adjacency_build(const mkg_graph* g, mkg_adjacency adj, int64_t* num_tasks, void* ws,
                                size_t ws_bytes, unsigned* err, mkg_stream st) {
  return mkg::adjacency_build(g, adj, num_tasks, ws, ws_bytes, err, S(st));
}
MKG_API int mkg_adjacency_set_factor(const mkg_graph* g, mkg_adjacency adj, const mkg_edge_factor* f,
                                     mkg_stream st) {
  return mkg::adjacency_set_factor(g, adj, f, S(st));
}
MKG_API int mkg_records_set_factor(mkg_adj_edge* records, int64_t count, int64_t num_facts, const mkg_edge_factor* f,
                                   mkg_stream st) {
  return mkg::records_set_factor(records, count, num_facts, f, S(st));
}

MKG_API int mkg_hop_count_messages(const mkg_graph* g, const mkg_frontier* f, const mkg_hop_params* p,
                                   int64_t* counts, unsigned* err, mkg_stream st) {
  return mkg::hop_count_messages(g, f, p, counts, err, S(st));
}
MKG_API size_t mkg_hop_forward_workspace_bytes(const mkg_hop_params* p, int64_t nnz) {
  return p ? mkg::hop_forward_workspace_bytes(p, nnz) : 0;
}
MKG_API int mkg_hop_forward(const mkg_graph* g, const mkg_frontier* f, const float* w, const mkg_edge_factor* ef,
                            const mkg_hop_params* p, void* ws, size_t ws_bytes, int64_t* counts, unsigned* err,
                            mkg_stream st) {
  return mkg::hop_forward(g, f, w, ef, p, ws, ws_bytes, counts, err, S(st));
}
MKG_API int mkg_hop_emit(const mkg_hop_params* p, int64_t nnz, const void* ws, size_t ws_bytes, int which,
                         int64_t count, int64_t* indices, float* values, int64_t* arg, mkg_stream st) {
  return mkg::hop_emit(p, nnz, ws, ws_bytes, which, count, indices, values, arg, S(st));
}
MKG_API size_t mkg_hop_backward_workspace_bytes(const mkg_hop_params* p, int64_t nnz) {
  return p ? mkg::hop_backward_workspace_bytes(p, nnz) : 0;
}
MKG_API int mkg_hop_backward(const mkg_graph* g, const mkg_frontier* f, const float* w, const mkg_edge_factor* ef,
                             const mkg_hop_params* p, const mkg_coo3* g_ori, const mkg_coo3* g_inv,
                             const mkg_coo3* g_ind, const mkg_coo3* out_ori, const int64_t* arg_ori,
                             const mkg_coo3* out_inv, const int64_t* arg_inv, const int32_t* fhead,
                             const int32_t* ftail, const int16_t* frel, float* grad_sp, float* grad_w,
                             float* grad_edge, void* ws, size_t ws_bytes, unsigned* err, mkg_stream st) {
  return mkg::hop_backward(g, f, w, ef, p, g_ori, g_inv, g_ind, out_ori, arg_ori, out_inv, arg_inv, fhead, ftail,
                           frel, grad_sp, grad_w, grad_edge, ws, ws_bytes, err, S(st));
}

MKG_API size_t mkg_proof_workspace_bytes(const mkg_proof_params* p) {
  return p ? mkg::proof_workspace_bytes(p) : 0;
}
MKG_API int mkg_proof_forward(const mkg_graph* g, const mkg_adjacency* adj, const int64_t* heads,
                              const float* w_hops, const mkg_proof_params* p, void* ws, size_t ws_bytes, float* out,
                              int64_t* messages, unsigned* err, mkg_stream st) {
  return mkg::proof_forward(g, adj, heads, w_hops, p, ws, ws_bytes, out, messages, err, S(st));
}
MKG_API int mkg_proof_backward(const mkg_graph* g, const mkg_adjacency* adj, const float* w_hops,
                               const mkg_proof_params* p, const mkg_edge_factor* ef, const float* grad_out,
                               float* grad_w_hops, float* grad_edge, void* ws, size_t ws_bytes, unsigned* err,
                               mkg_stream st) {
  return mkg::proof_backward(g, adj, w_hops, p, ef, grad_out, grad_w_hops, grad_edge, ws, ws_bytes, err, S(st));
}
MKG_API int mkg_proof_row_activity(const mkg_proof_params* p, const void* ws, size_t ws_bytes, int64_t h,
                                   uint8_t* flags, mkg_stream st) {
  return mkg::proof_row_activity(p, ws, ws_bytes, h, flags, S(st));
}
MKG_API size_t mkg_decode_workspace_bytes(const mkg_proof_params* p, int64_t topk) {
  return p ? mkg::decode_workspace_bytes(p, topk) : 0;
}
MKG_API int mkg_proof_decode_max(const mkg_graph* g, const mkg_adjacency* adj, const int64_t* heads,
                                 const float* w_hops, const mkg_proof_params* p, int64_t topk, float* out_scores,
                                 int64_t* tails, float* scores, int64_t* counts, void* ws, size_t ws_bytes,
                                 unsigned* err, mkg_stream st) {
  return mkg::proof_decode_max(g, adj, heads, w_hops, p, topk, out_scores, tails, scores, counts, ws, ws_bytes,
                               err, S(st));
}
MKG_API int mkg_decode_topk(const float* raw, int64_t B, int64_t E, int64_t topk, int64_t* tails, float* scores,
                            int64_t* counts, mkg_stream st) {
  return mkg::decode_topk(raw, B, E, topk, tails, scores, counts, S(st));
}
MKG_API size_t mkg_sparse_topk_workspace_bytes(int64_t nnz) { return mkg::sparse_topk_workspace_bytes(nnz); }
MKG_API int mkg_sparse_topk(const int64_t* keys, const float* vals, int64_t nnz, int64_t B, int64_t E, int64_t topk,
                            int64_t* tails, float* scores, int64_t* counts, void* ws, size_t ws_bytes,
                            mkg_stream st) {
  return mkg::sparse_topk(keys, vals, nnz, B, E, topk, tails, scores, counts, ws, ws_bytes, S(st));
}
MKG_API int mkg_segment_sum(const int64_t* seg_ptr, int64_t nseg, const float* values, float* out, mkg_stream st) {
  return mkg::segment_sum(seg_ptr, nseg, values, out, S(st));
}
MKG_API int mkg_segment_sum_ordered(const int64_t* seg_ptr, int64_t nseg, const float* values, float* out,
                                    mkg_stream st) {
  return mkg::segment_sum_ordered(seg_ptr, nseg, values, out, S(st));
}

MKG_API size_t mkg_rule_saved_bytes(const mkg_rule_params* p) { return mkg::rule_saved_bytes(p); }
MKG_API size_t mkg_rule_backward_workspace_bytes(const mkg_rule_params* p) {
  return mkg::rule_backward_workspace_bytes(p);
}
MKG_API size_t mkg_rule_softmax_workspace_bytes(const mkg_rule_params* p) {
  return mkg::rule_softmax_workspace_bytes(p);
}
MKG_API int mkg_rule_logits_forward(const mkg_rule_params* p, const float* emb, const float* w_ih,
                                    const float* w_hh, const float* bias, const float* w_lin, const float* b_lin,
                                    const int64_t* rel_u, float* logits_u, void* saved, size_t saved_bytes,
                                    unsigned* err, mkg_stream st) {
  return mkg::rule_logits_forward(p, emb, w_ih, w_hh, bias, w_lin, b_lin, rel_u, logits_u, saved, saved_bytes, err,
                                  S(st));
}
MKG_API int mkg_rule_logits_backward(const mkg_rule_params* p, const float* emb, const float* w_ih,
                                     const float* w_hh, const float* w_lin, const int64_t* rel_u, const void* saved,
                                     size_t saved_bytes, const float* grad_logits_u, float* grad_emb,
                                     float* grad_w_ih, float* grad_w_hh, float* grad_bias, float* grad_w_lin,
                                     float* grad_b_lin, void* ws, size_t ws_bytes, unsigned* err, mkg_stream st) {
  return mkg::rule_logits_backward(p, emb, w_ih, w_hh, w_lin, rel_u, saved, saved_bytes, grad_logits_u, grad_emb,
                                   grad_w_ih, grad_w_hh, grad_bias, grad_w_lin, grad_b_lin, ws, ws_bytes, err,
                                   S(st));
}
MKG_API int mkg_rule_softmax_forward(const mkg_rule_params* p, const float* logits_u, const int64_t* query_u,
                                     float* w_hops, unsigned* err, mkg_stream st) {
  return mkg::rule_softmax_forward(p, logits_u, query_u, w_hops, err, S(st));
}
MKG_API int mkg_rule_softmax_backward(const mkg_rule_params* p, const float* w_hops, const float* grad_w_hops,
                                      const int64_t* query_ptr, const int64_t* query_perm, float* grad_logits_u,
                                      void* ws, size_t ws_bytes, unsigned* err, mkg_stream st) {
  return mkg::rule_softmax_backward(p, w_hops, grad_w_hops, query_ptr, query_perm, grad_logits_u, ws, ws_bytes, err,
                                    S(st));
}

MKG_API size_t mkg_cap_index_workspace_bytes(const mkg_graph* g) { return mkg::cap_index_workspace_bytes(g); }
MKG_API int mkg_cap_index_sizes(const mkg_graph* g, int64_t cap, int64_t* sizes_out, void* ws, size_t ws_bytes,
                                mkg_stream st) {
  return mkg::cap_index_sizes(g, cap, sizes_out, ws, ws_bytes, S(st));
}
MKG_API int mkg_cap_index_build(const mkg_graph* g, const mkg_adjacency* adj, const mkg_cap_index* index, void* ws,
                                size_t ws_bytes, unsigned* err, mkg_stream st) {
  return mkg::cap_index_build(g, adj, index, ws, ws_bytes, err, S(st));
}
