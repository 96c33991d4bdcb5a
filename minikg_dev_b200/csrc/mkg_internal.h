// Internal entry points behind the C ABI (one namespace, one definition per .cu file).
#pragma once

#include <cuda_runtime.h>

#include "minikg_b200.h"

namespace mkg {

// mkg_graph.cu
size_t csr_build_workspace_bytes(int64_t T, int64_t E, int64_t R);
int csr_build(const int32_t* head, const int32_t* rel, const int32_t* tail, int64_t T, int64_t E, int64_t R,
              mkg_csr_dir_out ori, mkg_csr_dir_out inv, int64_t* num_groups, void* ws, size_t ws_bytes,
              unsigned* err, cudaStream_t st);
size_t ind2ptr_workspace_bytes(int64_t size);
int ind2ptr(const int64_t* index, int64_t n, int64_t size, int64_t* ptr, void* ws, size_t ws_bytes,
            unsigned* err, cudaStream_t st);
int fact_table(const mkg_graph* g, int32_t* head, int32_t* tail, int16_t* rel, unsigned* err, cudaStream_t st);
int64_t adjacency_max_tasks(int64_t E, int64_t T);
size_t adjacency_workspace_bytes(int64_t E);
int adjacency_build(const mkg_graph* g, mkg_adjacency adj, int64_t* num_tasks, void* ws, size_t ws_bytes,
                    unsigned* err, cudaStream_t st);
int adjacency_set_factor(const mkg_graph* g, mkg_adjacency adj, const mkg_edge_factor* f, cudaStream_t st);
int records_set_factor(mkg_adj_edge* recs, int64_t count, int64_t num_facts, const mkg_edge_factor* f,
                       cudaStream_t st);
size_t cap_index_workspace_bytes(const mkg_graph* g);
int cap_index_sizes(const mkg_graph* g, int64_t cap, int64_t* sizes, void* ws, size_t ws_bytes, cudaStream_t st);
int cap_index_build(const mkg_graph* g, const mkg_adjacency* adj, const mkg_cap_index* ix, void* ws,
                    size_t ws_bytes, unsigned* err, cudaStream_t st);

// mkg_hop.cu
int hop_count_messages(const mkg_graph* g, const mkg_frontier* fr, const mkg_hop_params* p, int64_t* counts_out,
                       unsigned* err, cudaStream_t st);
size_t hop_forward_workspace_bytes(const mkg_hop_params* p, int64_t nnz);
int hop_forward(const mkg_graph* g, const mkg_frontier* fr, const float* w, const mkg_edge_factor* ef,
                const mkg_hop_params* p, void* ws, size_t ws_bytes, int64_t* counts_out, unsigned* err,
                cudaStream_t st);
int hop_emit(const mkg_hop_params* p, int64_t nnz, const void* ws, size_t ws_bytes, int which, int64_t count,
             int64_t* indices, float* values, int64_t* arg, cudaStream_t st);
size_t hop_backward_workspace_bytes(const mkg_hop_params* p, int64_t nnz);
int hop_backward(const mkg_graph* g, const mkg_frontier* fr, const float* w, const mkg_edge_factor* ef,
                 const mkg_hop_params* p, const mkg_coo3* g_ori, const mkg_coo3* g_inv, const mkg_coo3* g_ind,
                 const mkg_coo3* out_ori, const int64_t* arg_ori, const mkg_coo3* out_inv, const int64_t* arg_inv,
                 const int32_t* fhead, const int32_t* ftail, const int16_t* frel, float* grad_sp, float* grad_w,
                 float* grad_edge, void* ws, size_t ws_bytes, unsigned* err, cudaStream_t st);

// mkg_proof.cu
size_t proof_workspace_bytes(const mkg_proof_params* p);
int proof_forward(const mkg_graph* g, const mkg_adjacency* adj, const int64_t* heads, const float* w_hops,
                  const mkg_proof_params* p, void* ws, size_t ws_bytes, float* out, int64_t* messages_out,
                  unsigned* err, cudaStream_t st);
int proof_backward(const mkg_graph* g, const mkg_adjacency* adj, const float* w_hops, const mkg_proof_params* p,
                   const mkg_edge_factor* ef, const float* grad_out, float* grad_w_hops, float* grad_edge, void* ws,
                   size_t ws_bytes, unsigned* err, cudaStream_t st);
int proof_row_activity(const mkg_proof_params* p, const void* ws, size_t ws_bytes, int64_t h, uint8_t* flags,
                       cudaStream_t st);
size_t decode_workspace_bytes(const mkg_proof_params* p, int64_t topk);
int proof_decode_max(const mkg_graph* g, const mkg_adjacency* adj, const int64_t* heads, const float* w_hops,
                     const mkg_proof_params* p, int64_t topk, float* out_scores, int64_t* tails, float* scores,
                     int64_t* counts, void* ws, size_t ws_bytes, unsigned* err, cudaStream_t st);
int decode_topk(const float* raw, int64_t B, int64_t E, int64_t topk, int64_t* tails, float* scores,
                int64_t* counts, cudaStream_t st);
size_t sparse_topk_workspace_bytes(int64_t nnz);
int sparse_topk(const int64_t* keys, const float* vals, int64_t nnz, int64_t B, int64_t E, int64_t topk,
                int64_t* tails, float* scores, int64_t* counts, void* ws, size_t ws_bytes, cudaStream_t st);
int segment_sum_ordered(const int64_t* seg_ptr, int64_t nseg, const float* values, float* out, cudaStream_t st);
int segment_sum(const int64_t* seg_ptr, int64_t nseg, const float* values, float* out, cudaStream_t st);

// mkg_rules.cu
size_t rule_saved_bytes(const mkg_rule_params* p);
size_t rule_backward_workspace_bytes(const mkg_rule_params* p);
size_t rule_softmax_workspace_bytes(const mkg_rule_params* p);
int rule_logits_forward(const mkg_rule_params* p, const float* emb, const float* w_ih, const float* w_hh,
                        const float* bias, const float* w_lin, const float* b_lin, const int64_t* rel_u,
                        float* logits_u, void* saved, size_t saved_bytes, unsigned* err, cudaStream_t st);
int rule_logits_backward(const mkg_rule_params* p, const float* emb, const float* w_ih, const float* w_hh,
                         const float* w_lin, const int64_t* rel_u, const void* saved, size_t saved_bytes,
                         const float* grad_logits_u, float* grad_emb, float* grad_w_ih, float* grad_w_hh,
                         float* grad_bias, float* grad_w_lin, float* grad_b_lin, void* ws, size_t ws_bytes,
                         unsigned* err, cudaStream_t st);
int rule_softmax_forward(const mkg_rule_params* p, const float* logits_u, const int64_t* query_u, float* w_hops,
                         unsigned* err, cudaStream_t st);
int rule_softmax_backward(const mkg_rule_params* p, const float* w_hops, const float* grad_w_hops,
                          const int64_t* query_ptr, const int64_t* query_perm, float* grad_logits_u, void* ws,
                          size_t ws_bytes, unsigned* err, cudaStream_t st);

}  // namespace mkg
