/*
 * minikg_b200 — C ABI of the B200 (sm_100a) relation-typed sparse hop library.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream, returns an
 * int status (MKG_OK = 0) and leaves a message for mkg_last_error() on failure.  The
 * library never allocates device memory: callers pass output buffers and a workspace
 * sized by the matching *_workspace_bytes() query.  Kernels that meet a bad index do
 * not fault; they skip the access and set a bit in the caller's device error word.
 *
 * Each declaration names the reference interface (majh3/miniKG_dev) it replaces.
 */
#ifndef MINIKG_B200_H
#define MINIKG_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* mkg_stream; /* a cudaStream_t; NULL = legacy default stream */

enum {
  MKG_OK = 0,
  MKG_ERR_ARG = 1,       /* bad shape / size / pointer / parameter */
  MKG_ERR_INDEX = 2,     /* a device kernel reported an out-of-range index */
  MKG_ERR_CAPACITY = 3,  /* workspace or output smaller than required */
  MKG_ERR_CUDA = 4,      /* a CUDA runtime call failed */
  MKG_ERR_TIMEOUT = 5,   /* a bounded device wait gave up */
  MKG_ERR_UNSUPPORTED = 6
};

enum { MKG_MASK_NONE = 0, MKG_MASK_U8 = 1, MKG_MASK_F32 = 2 };

/* bits of the device error word */
enum {
  MKG_DEV_BAD_ENTRY = 1u,  /* frontier (batch, level, entity) outside [B, L, E] */
  MKG_DEV_BAD_COL = 2u,    /* CSR column / neighbour outside [0, E) */
  MKG_DEV_BAD_FACT = 4u,   /* CSR order / fact id outside [0, T) */
  MKG_DEV_BAD_KEY = 8u,    /* gradient COO key outside [B, L, E] */
  MKG_DEV_BAD_REL = 16u,   /* relation id outside [0, R) */
  MKG_DEV_TIMEOUT = 32u,   /* a bounded wait inside a kernel gave up */
  MKG_DEV_TABLE_FULL = 64u, /* a message hash table ran out of slots (msg_bound too small) */
  MKG_DEV_BAD_RULE_INDEX = 128u /* rule producer: relation outside [0, n) or query map outside [0, U) */
};

/* One direction of the reference CSR pair (fastlog_kernel.py:403-410 tuple order). */
typedef struct mkg_csr_dir {
  const int32_t* row_ptr;          /* [E+1] */
  const int32_t* col_ind;          /* [T]   neighbour per CSR position */
  const int16_t* r_ind;            /* [T]   relation per CSR position */
  const int32_t* order;            /* [T]   original fact id per CSR position */
  const int32_t* row_group_ptr;    /* [E+1] */
  const int16_t* group_rel;        /* [G] */
  const int32_t* group_edge_start; /* [G] */
  const int32_t* group_edge_count; /* [G] */
  int64_t num_groups;
} mkg_csr_dir;

typedef struct mkg_graph {
  int64_t num_entities;  /* E */
  int64_t num_relations; /* R (relation ids lie in [0, R)) */
  int64_t num_facts;     /* T */
  mkg_csr_dir ori;       /* rows = head, sorted by (head, rel, fact id) */
  mkg_csr_dir inv;       /* rows = tail, sorted by (tail, rel, fact id) */
} mkg_graph;

/* Edge factor m = bool(mask[f]) * score(f) (fastlog.cu:2303-2309). */
typedef struct mkg_edge_factor {
  const void* mask;           /* NULL: all facts on */
  int32_t mask_kind;          /* MKG_MASK_* */
  int64_t mask_numel;         /* T, or 1 to broadcast one value to every fact */
  const float* edge_weight;   /* [T] or NULL */
  int64_t edge_weight_numel;  /* 0: no score factor */
  int32_t is_score;           /* 1: score = weight; 0: score = sigmoid(weight * scale) */
  float scale;
} mkg_edge_factor;

/* Sparse [B, L, E] frontier in COO (the op's sp_batch/sp_level/sp_entity/sp_value). */
typedef struct mkg_frontier {
  const int64_t* batch;
  const int64_t* level;
  const int64_t* entity;
  const float* value;
  int64_t nnz;
} mkg_frontier;

/* Sparse [B, L, E] gradient / output in COO: indices [3, nnz] row-major, values [nnz]. */
typedef struct mkg_coo3 {
  const int64_t* indices;
  const float* values;
  int64_t nnz;
} mkg_coo3;

const char* mkg_last_error(void);
int mkg_abi_version(void);

/* ------------------------------------------------------------------ graph build */

/* Caller-allocated outputs of mkg_csr_build; group arrays are sized T (upper bound). */
typedef struct mkg_csr_dir_out {
  int32_t* row_ptr;
  int32_t* col_ind;
  int16_t* r_ind;
  int32_t* order;
  int32_t* row_group_ptr;
  int16_t* group_rel;
  int32_t* group_edge_start;
  int32_t* group_edge_count;
} mkg_csr_dir_out;

/* Replaces build_csr_structure (src/fastlog_kernel/fastlog_kernel.py:371-411) and its
 * helpers _build_group_metadata (:354-368) / _ind2ptr_cpu (:346-351): device radix
 * sort to a stable (row, rel, fact id) order for both directions.  Writes the two
 * group counts to num_groups_out (device int64[2]). */
size_t mkg_csr_build_workspace_bytes(int64_t num_facts, int64_t num_entities, int64_t num_relations);
int mkg_csr_build(const int32_t* head, const int32_t* rel, const int32_t* tail, int64_t num_facts,
                  int64_t num_entities, int64_t num_relations, mkg_csr_dir_out ori,
                  mkg_csr_dir_out inv, int64_t* num_groups_out, void* workspace,
                  size_t workspace_bytes, unsigned* dev_err, mkg_stream stream);

/* Replaces ind2ptr (src/fastlog_kernel/source/fastlog.cpp:9-16, fastlog.h:13):
 * ptr[0..size] = exclusive prefix of the per-row counts of index[0..n), ptr[size] = n. */
size_t mkg_ind2ptr_workspace_bytes(int64_t size);
int mkg_ind2ptr(const int64_t* index, int64_t n, int64_t size, int64_t* ptr, void* workspace,
                size_t workspace_bytes, unsigned* dev_err, mkg_stream stream);

/* ind2ptr for callers that cannot allocate device memory (for example a C or FFI host
 * holding only the device pointers it was given): same inputs and output as mkg_ind2ptr,
 * no workspace argument.  No counterpart in the reference.  Its scratch is one static
 * device array of about 8.3 MiB that every GPU loading the library keeps until exit;
 * size is limited to MKG_NOALLOC_MAX_ROWS rows (larger: MKG_ERR_CAPACITY).  Every call made
 * outside a stream capture looks the array's device address up again (it can move after a
 * cudaDeviceReset); a call inside a capture reuses the last such address, so the first call
 * on a device should come before any stream capture.  Calls that overlap on the GPU share
 * the array and race. */
#define MKG_NOALLOC_MAX_ROWS (1 << 20)
int mkg_ind2ptr_noalloc(const int64_t* index, int64_t n, int64_t size, int64_t* ptr, unsigned* dev_err,
                        mkg_stream stream);

/* Per-fact endpoints recovered from the ori CSR (used by the argmax backward):
 * fact_head[f], fact_tail[f], fact_rel[f].  No reference counterpart: the reference
 * keeps them per raw message (meta_entry / meta_rel, fastlog.cu:2314-2317). */
int mkg_fact_table(const mkg_graph* g, int32_t* fact_head, int32_t* fact_tail, int16_t* fact_rel,
                   unsigned* dev_err, mkg_stream stream);

/* Merged neighbour lists of the fused engine.  pull row d = every message that can reach
 * d: facts with tail d (neighbour = head, channel = rel) then facts with head d
 * (neighbour = tail, channel = R + rel); push row s = every message s can send.  Records
 * are 16 bytes: {neighbour, channel, fact id, edge factor}. */
typedef struct mkg_adj_edge {
  int32_t nbr;
  int32_t channel;
  int32_t fact;
  float factor;
} mkg_adj_edge;

/* Rows are cut into tasks of at most 64 records: int32 quadruples {row, begin, end, flags}
 * (flags: 1 = first task of its row, 2 = the row spans several tasks). */
typedef struct mkg_adjacency {
  int32_t* pull_ptr;      /* [E+1] */
  mkg_adj_edge* pull;     /* [2T] */
  int32_t* push_ptr;      /* [E+1] */
  mkg_adj_edge* push;     /* [2T] */
  int32_t* pull_tasks;    /* [4 * mkg_adjacency_max_tasks(E, T)] */
  int64_t num_pull_tasks; /* filled by the caller from num_tasks_out[0] */
  int32_t* push_tasks;    /* [4 * mkg_adjacency_max_tasks(E, T)] */
  int64_t num_push_tasks; /* filled by the caller from num_tasks_out[1] */
} mkg_adjacency;

int64_t mkg_adjacency_max_tasks(int64_t num_entities, int64_t num_facts);
size_t mkg_adjacency_workspace_bytes(int64_t num_entities);
/* Builds both neighbour lists and their task lists; writes the two task counts to
 * num_tasks_out (device int64[2]).  No reference counterpart (the reference pushes raw
 * messages per frontier entry, fastlog.cu:2197-2323). */
int mkg_adjacency_build(const mkg_graph* g, mkg_adjacency adj, int64_t* num_tasks_out, void* workspace,
                        size_t workspace_bytes, unsigned* dev_err, mkg_stream stream);
/* Rewrites the factor field of every record from the current mask / edge scores; a list
 * whose pointer (adj.pull or adj.push) is NULL is left as it is.  mkg_records_set_factor does
 * the same for any record array (e.g. a rank's push records of its own destinations). */
int mkg_adjacency_set_factor(const mkg_graph* g, mkg_adjacency adj, const mkg_edge_factor* f,
                             mkg_stream stream);
int mkg_records_set_factor(mkg_adj_edge* records, int64_t count, int64_t num_facts, const mkg_edge_factor* f,
                           mkg_stream stream);

/* Edge-cap index of the fused engine for one cap value (0 .. MKG_DENSE_CAP_MAX).  The
 * reference caps every frontier entry (b, l, s) per direction at `cap` messages with the
 * 256-bucket rule of fastlog.cu:2092-2195, 2273-2298: the relation groups of s's CSR row are
 * bucketed by the rule weight w[b, l, channel]; groups above the threshold bucket take all
 * their edges, groups below take none, threshold-bucket groups take in group order what is
 * left of the cap, each its first edges in CSR order.  Only rows longer than the cap are
 * affected ("capped rows"); every relation group of a capped row gets one row of a per-hop
 * take table [num_groups, B*L] (uint8: edges taken per column), and every pull / push record
 * sent by a capped row points at its group's row and its position inside the group. */
#define MKG_DENSE_CAP_MAX 255
typedef struct mkg_cap_index {
  int64_t cap;
  int64_t num_slots;             /* capped (entity, direction) rows */
  int64_t num_groups;            /* relation groups of the capped rows: rows of the take table */
  const int32_t* slot_entity;    /* [num_slots] */
  const int32_t* slot_dir;       /* [num_slots] 0: ori (rows = heads), 1: inv (rows = tails) */
  const int32_t* slot_group;     /* [num_slots] take-table row of the slot's first group */
  const int32_t* pull_cap;       /* [2 * records] per pull record: (take row or -1, position in group) */
  const int32_t* push_cap;       /* [2 * records] the same per push record */
  const int32_t* capped_degree;  /* [E] min(out-degree ori, cap) + min(out-degree inv, cap) */
} mkg_cap_index;

/* Writes (num_slots, num_groups) of the index for `cap` to sizes_out (device int64[2]). */
size_t mkg_cap_index_workspace_bytes(const mkg_graph* g);
int mkg_cap_index_sizes(const mkg_graph* g, int64_t cap, int64_t* sizes_out, void* workspace,
                        size_t workspace_bytes, mkg_stream stream);
/* Fills the caller-allocated arrays of `index` (sizes from mkg_cap_index_sizes; the records of
 * `adj` from mkg_adjacency_build).  No reference counterpart: the reference decides the cap
 * per frontier entry while it expands messages (fastlog.cu:2114-2323). */
int mkg_cap_index_build(const mkg_graph* g, const mkg_adjacency* adj, const mkg_cap_index* index,
                        void* workspace, size_t workspace_bytes, unsigned* dev_err, mkg_stream stream);

/* ------------------------------------------------------------------ per-hop op */

typedef struct mkg_hop_params {
  int64_t B, L, E;
  int64_t r_size;      /* channel offset of the inverse direction (= R) */
  int64_t n;           /* channels of w: w is [B, L, n], identity channel n-1 */
  int32_t wot_i;       /* 1: identity channel contributes zeros */
  int32_t agg_mode;    /* 0 sum, 1 max with argmax */
  int64_t topk_edges;  /* per-entry edge cap; >= 2^60 means uncapped */
  /* Destination range [dst_lo, dst_hi): only messages whose destination entity (the
   * identity channel's is the entry itself) lies in it are produced, and the output key
   * space is B x L x (dst_hi - dst_lo).  Caps are still decided on the whole CSR row, so
   * the union over a partition of [0, E) equals the full-range output.  dst_hi <= dst_lo
   * (e.g. both 0) means [0, E).  No counterpart in the reference (single GPU); used by the
   * destination-partitioned multi-GPU hop.  agg_mode 1 backward needs the full range. */
  int64_t dst_lo, dst_hi;
  /* Upper bound on the messages of one direction (ori or inv) of this hop, e.g. the larger
   * count written by mkg_hop_count_messages; 0 = unknown.  Messages are reduced in a dense
   * slab indexed by the output key unless the bound is far below the key space
   * (32 * msg_bound < B * L * extent): then in open-addressing hash tables of
   * 2^ceil(log2(2 * bound)) slots, sorted by key for the output.  The forward, emit and
   * backward calls of one hop must all see the same value. */
  int64_t msg_bound;
  /* 0: choose as above; 1: always the dense slab; 2: hash tables (needs msg_bound >= the
   * real message count of each direction, else MKG_DEV_TABLE_FULL). */
  int64_t accum;
  /* 1 (agg_mode 0 only): ori, inv and ind are reduced into one output (which = 0; outputs
   * 1 and 2 are empty), i.e. sum_sparse3d_concat(ori, inv, ind) of the hop loop
   * (src/fastlog_bridge.py:26-42) done by the op; msg_bound must then bound ori + inv +
   * entries.  The backward takes that output's gradient as g_ori (g_inv, g_ind ignored). */
  int64_t merge_outputs;
} mkg_hop_params;

/* Exact message counts of one hop (no counterpart in the reference, whose count kernels
 * fastlog.cu:2721-2730 feed a device cumsum): counts_out[0] / [1] (device int64) = the
 * frontier's ori / inv messages, per entry min(out-degree, cap) (the 256-bucket cap takes
 * exactly cap edges of a longer row; cap <= 0 takes none).  Destination ranges do not
 * change the count (every rank of a partition walks the same messages). */
int mkg_hop_count_messages(const mkg_graph* g, const mkg_frontier* f, const mkg_hop_params* p,
                           int64_t* counts_out, unsigned* dev_err, mkg_stream stream);

/* Forward of one hop, coalesced: replaces fastlog_forward_sparse3d_topk_cuda
 * (src/fastlog_kernel/source/fastlog.h:78-93, fastlog.cu:2678-2806) together with the
 * torch coalescing that follows it (fastlog_kernel.py:951-966, _coalesce_sparse3d_reduce
 * :81-104, _coalesce_sparse3d_max_with_arg :107-150).  Raw messages are never
 * materialised: they are reduced in HBM slabs indexed by the key b*L*E + l*E + e.
 * Writes the output sizes (ori, inv, ind) to counts_out (device int64[3]).  The
 * workspace must stay alive and unmodified until mkg_hop_emit has run for all three. */
size_t mkg_hop_forward_workspace_bytes(const mkg_hop_params* p, int64_t nnz);
int mkg_hop_forward(const mkg_graph* g, const mkg_frontier* f, const float* w,
                    const mkg_edge_factor* ef, const mkg_hop_params* p, void* workspace,
                    size_t workspace_bytes, int64_t* counts_out, unsigned* dev_err, mkg_stream stream);

/* Writes output `which` (0 ori, 1 inv, 2 ind) as sorted coalesced COO: indices [3, count]
 * (int64), values [count]; for agg_mode 1 and which < 2 also arg_fact [count] = fact id of
 * the argmax message (smallest fact id among equal maxima).  nnz = the forward's frontier size. */
int mkg_hop_emit(const mkg_hop_params* p, int64_t nnz, const void* workspace, size_t workspace_bytes,
                 int which, int64_t count, int64_t* indices, float* values, int64_t* arg_fact,
                 mkg_stream stream);

/* Backward of one hop: replaces fastlog_backward_sparse3d_topk_cuda (fastlog.h:123-134,
 * fastlog.cu:3037-3109) for agg_mode 0 and fastlog_backward_sparse3d_topk_aligned_cuda
 * (fastlog.h:136-145, fastlog.cu:3111-3181) with _align_sparse_grad_to_raw_argmax
 * (fastlog_kernel.py:153-167) for agg_mode 1, plus the edge-score gradient of
 * fastlog_kernel.py:1032-1098.  grad_ori / grad_inv / grad_ind are the incoming COO
 * gradients; for agg_mode 1, out_ori / out_inv are the forward outputs (indices) with
 * their arg_fact arrays.  Writes grad_sp [nnz], grad_w [B, L, n] and, when not NULL,
 * grad_edge [T] (all overwritten). */
size_t mkg_hop_backward_workspace_bytes(const mkg_hop_params* p, int64_t nnz);
int mkg_hop_backward(const mkg_graph* g, const mkg_frontier* f, const float* w,
                     const mkg_edge_factor* ef, const mkg_hop_params* p, const mkg_coo3* grad_ori,
                     const mkg_coo3* grad_inv, const mkg_coo3* grad_ind, const mkg_coo3* out_ori,
                     const int64_t* arg_ori, const mkg_coo3* out_inv, const int64_t* arg_inv,
                     const int32_t* fact_head, const int32_t* fact_tail, const int16_t* fact_rel,
                     float* grad_sp, float* grad_w, float* grad_edge, void* workspace,
                     size_t workspace_bytes, unsigned* dev_err, mkg_stream stream);

/* ------------------------------------------------------------------ fused hop loop */

typedef struct mkg_proof_params {
  int64_t B, L, E, R;
  int64_t hops;
  int64_t topk_edges;      /* per-entry edge cap (>= 2^60: uncapped) */
  float state_threshold;   /* >0: drop normalised state values below it after each hop */
  int32_t reserved;
  /* Optional caller-owned cudaEvent_t arrays of 2*hops events each (NULL: none).  The
   * library records event 2h before and 2h+1 after the pull kernel of hop h (forward) /
   * the transposed pull of hop h (backward), on the call's stream. */
  void* const* fwd_events;
  void* const* bwd_events;
  /* Required when topk_edges < 2^60 (then 0 <= topk_edges <= MKG_DENSE_CAP_MAX): the cap
   * index built for topk_edges.  Messages of capped rows not taken under the cap are left
   * out of every hop, forward and backward, and of the message counts. */
  const mkg_cap_index* cap_index;
} mkg_proof_params;

/* The whole hop loop of kernel_sparse_scores (proof.py:467-614, dropout off, no entity
 * pruning) on a dense entity-major state: per hop the op, sum_sparse3d_concat
 * (fastlog_bridge.py:26-42), normalize_sparse3d(.., 0, "mass") (drum.py:31-51); then
 * sum_sp_3d (fastlog_bridge.py:17-23) into out [B, E].  w_hops is [hops, B, L, 2R+1].
 * The workspace keeps every hop's state for mkg_proof_backward; messages_out (device
 * int64[hops], may be NULL) receives the per-hop message counts. */
size_t mkg_proof_workspace_bytes(const mkg_proof_params* p);
int mkg_proof_forward(const mkg_graph* g, const mkg_adjacency* adj, const int64_t* heads,
                      const float* w_hops, const mkg_proof_params* p, void* workspace,
                      size_t workspace_bytes, float* out, int64_t* messages_out, unsigned* dev_err,
                      mkg_stream stream);

/* Row activity of the state that entered hop h of the last mkg_proof_forward /
 * mkg_proof_decode_max run in this workspace: row_flags[e] = 1 when entity e holds a
 * non-zero value for some (query, rule).  Used to count the compulsory bytes of a hop. */
int mkg_proof_row_activity(const mkg_proof_params* p, const void* workspace, size_t workspace_bytes, int64_t h,
                           uint8_t* row_flags, mkg_stream stream);

/* Gradients of mkg_proof_forward: grad_out [B, E] (only entries where out != 0 count, as
 * for the reference's sparse result) -> grad_w_hops [hops, B, L, n] and, when not NULL,
 * grad_edge [T] (edge-score gradient, fastlog_kernel.py:1032-1098).  Outputs are
 * overwritten.  Needs the workspace of the matching forward. */
int mkg_proof_backward(const mkg_graph* g, const mkg_adjacency* adj, const float* w_hops,
                       const mkg_proof_params* p, const mkg_edge_factor* ef, const float* grad_out,
                       float* grad_w_hops, float* grad_edge, void* workspace, size_t workspace_bytes,
                       unsigned* dev_err, mkg_stream stream);

/* Max-aggregation hop loop and decode (src/model_mmDRUM_kernel_sp.py:388-445 with the
 * "max" transition: op agg_mode 1 -> sparse3d_max(ind, ori, inv) -> norm_sp_3d between
 * hops, norm_sp_3d_max after the last), then bound_sparse_scores (proof.py:642-649) and
 * the decode order of ordered_tail_scores (decode_core.py:350-363): per query the
 * `topk` best (score desc, tail asc).  out_scores [B, E] receives the raw max scores;
 * tails [B, topk] (-1 padded), scores [B, topk], counts [B]. */
size_t mkg_decode_workspace_bytes(const mkg_proof_params* p, int64_t topk);
int mkg_proof_decode_max(const mkg_graph* g, const mkg_adjacency* adj, const int64_t* heads,
                         const float* w_hops, const mkg_proof_params* p, int64_t topk,
                         float* out_scores, int64_t* tails, float* scores, int64_t* counts,
                         void* workspace, size_t workspace_bytes, unsigned* dev_err, mkg_stream stream);

/* Decode ordering alone on a dense [B, E] raw score matrix (entries != 0 are candidates):
 * bound 1 - exp(-max(x, 0)), order (score desc, tail asc), keep topk per row.  Replaces
 * bound_sparse_scores + sparse_candidate_rows + ordered_tail_scores (proof.py:642-649,
 * 729-758, decode_core.py:350-363). */
int mkg_decode_topk(const float* raw, int64_t B, int64_t E, int64_t topk, int64_t* tails,
                    float* scores, int64_t* counts, mkg_stream stream);

/* The same decode ordering on a sparse [B, E] result: keys [nnz] (b * E + e, ascending) and
 * raw values [nnz]; every stored entry is a candidate (as proof.py:729-758 takes the rows of
 * the sparse tensor).  One block per query finds its row by binary search; keys of rows
 * outside [0, B) are ignored.  tails [B, topk] (-1 padded), scores [B, topk], counts [B];
 * topk in [1, 1024].  The workspace (mkg_sparse_topk_workspace_bytes(nnz) bytes) holds every
 * entry's candidate key, formed once. */
size_t mkg_sparse_topk_workspace_bytes(int64_t nnz);
int mkg_sparse_topk(const int64_t* keys, const float* vals, int64_t nnz, int64_t B, int64_t E, int64_t topk,
                    int64_t* tails, float* scores, int64_t* counts, void* workspace, size_t workspace_bytes,
                    mkg_stream stream);

/* out[s] = values[seg_ptr[s]] + values[seg_ptr[s] + 1] + ... + values[seg_ptr[s+1] - 1],
 * added one by one in index order in fp32 (device pointers; seg_ptr [nseg + 1], int64).
 * The row sums of norm_sp_3d (src/model_mmDRUM_kernel_sp.py:39-52) over a coalesced COO
 * whose (b, l) rows are contiguous, in the order the reference's CPU index_put_
 * accumulates them, so the max-aggregation decode stays bit-exact on sparse frontiers. */
int mkg_segment_sum_ordered(const int64_t* seg_ptr, int64_t nseg, const float* values, float* out,
                            mkg_stream stream);

/* out[s] = sum of values[seg_ptr[s] .. seg_ptr[s+1]) (fp32, tree order; one block per
 * segment): the row sums of normalize_sparse3d (drum.py:31-50) and of its gradient on a
 * key-sorted sparse state, without atomics on the few row bins.  No reference counterpart
 * (the reference coalesces and index_puts). */
int mkg_segment_sum(const int64_t* seg_ptr, int64_t nseg, const float* values, float* out, mkg_stream stream);

/* ------------------------------------------------------------ key-slab hop engine */

/* The uncapped sum hop of kernel_sparse_scores (proof.py:569-609: the op of
 * FastLogFunctionSparse3DTopK forward, fastlog.cu:2678-2806 with topk_edges uncapped, then the
 * coalescing of _coalesce_sparse3d_reduce, fastlog_kernel.py:81-104, and sum_sparse3d_concat,
 * fastlog_bridge.py:26-42) for large graphs with sparse frontiers.  Output keys of one call
 * lie in a window: (b, l) rows [row0, row0 + nrows) x destination entities [lo, lo + extent)
 * of a key space (row) * E + e.  A *store* of mkg_slab_store_bytes(nrows * extent) bytes
 * holds one fp32 slot per key and a touched bit per slot; the caller zero-fills it once and
 * every mkg_slab_emit / clearing mkg_slab_take leaves what it read at zero again.  Slots are
 * entity-major (slot (e - lo) * nrows + (row - row0)), and keys come out of mkg_slab_emit in
 * that order: ascending entity, then ascending row ("entity-major order").  A frontier or a
 * key list spanning several row windows is passed whole to each window's call; entries of
 * other rows are skipped by mkg_slab_expand and mkg_slab_expand_backward.  A destination range
 * may also be cut into tiles, each with a push list restricted to its destinations, walked
 * tile by tile in one launch (mkg_slab_expand_tiles: a tile's updates then stay in L2); a tile
 * may also be given a window of its own, and mkg_slab_put and mkg_slab_take given
 * MKG_SLAB_SKIP_OUTSIDE skip the keys outside their window (other rows or other tiles). */
#define MKG_SLAB_SKIP_OUTSIDE 16
typedef struct mkg_slab_window {
  int64_t E;       /* entities of the key space */
  int64_t row0;    /* first row (b * L + l, or b for [B, E] keys) of the window */
  int64_t nrows;   /* rows in the window */
  int64_t lo;      /* first destination entity */
  int64_t extent;  /* destination entities [lo, lo + extent) */
} mkg_slab_window;

size_t mkg_slab_store_bytes(int64_t slots);
size_t mkg_slab_expand_workspace_bytes(int64_t nnz);
/* Adds every message of the frontier entries in the window's rows (keys (b * L + l) * E + s
 * with values, in any order; entity-major order keeps the atomics of neighbouring entries in
 * the same sectors) to the store: for each record of push row s (mkg_adjacency.push, or a push
 * list restricted to destinations in [lo, lo + extent)) the value (x * w[b, l, channel]) *
 * factor at key (b, l, neighbour), plus (identity != 0) x * w[b, l, n - 1] at (b, l, s).
 * w is [B * L, n].  Zero-valued messages are left out (the hop loop drops zeros after its
 * normalisation).  agg_mode 0 adds the messages of a key (the sum hop, see above); agg_mode 1
 * keeps their maximum (the values of the max-aggregation hop, op agg_mode 1 followed by
 * sparse3d_max(ind, ori, inv), model_mmDRUM_kernel_sp.py:237-270, 388-445; the values must be
 * non-negative, as the loop's are).  row_sums (agg_mode 0, may be NULL): [nrows] fp64, each
 * window row's added message values are added to row_sums[r] (the column sums of
 * normalize_sparse3d, drum.py:31-51: the sum of the row's output values, summed exactly in
 * fp64 from the messages rather than from their fp32 per-key totals). */
int mkg_slab_expand(const int32_t* push_ptr, const mkg_adj_edge* push, const int64_t* keys, const float* vals,
                    int64_t nnz, const float* w, int64_t n, int32_t identity, int32_t agg_mode,
                    const mkg_slab_window* win, void* store, double* row_sums, void* workspace,
                    size_t workspace_bytes, unsigned* dev_err, mkg_stream stream);
/* mkg_slab_expand over the push lists of ntiles destination tiles (1..MKG_SLAB_MAX_TILES) in
 * one launch: push_ptrs / pushes are host arrays of the tiles' device lists (each [E + 1] /
 * records restricted to the tile's destinations; together every record of the window's range
 * once).  Work runs tile by tile, so the store sectors being updated at any time are one
 * tile's.  The identity messages (identity != 0) are added once, with tile 0.  Workspace:
 * mkg_slab_expand_workspace_bytes(nnz * ntiles). */
#define MKG_SLAB_MAX_TILES 8
int mkg_slab_expand_tiles(int32_t ntiles, const int32_t* const* push_ptrs, const mkg_adj_edge* const* pushes,
                          const int64_t* keys, const float* vals, int64_t nnz, const float* w, int64_t n,
                          int32_t identity, int32_t agg_mode, const mkg_slab_window* win, void* store,
                          double* row_sums, void* workspace, size_t workspace_bytes, unsigned* dev_err,
                          mkg_stream stream);
/* Number of touched keys in the store -> count_out (device int64).  The workspace (also read
 * by mkg_slab_emit) keeps per-tile offsets. */
size_t mkg_slab_collect_workspace_bytes(int64_t slots);
int mkg_slab_count(const mkg_slab_window* win, const void* store, void* workspace, size_t workspace_bytes,
                   int64_t* count_out, mkg_stream stream);
/* Writes the touched keys in entity-major order (global keys (row0 + r) * E + lo + e) with
 * their values and clears them in the store. */
int mkg_slab_emit(const mkg_slab_window* win, void* store, const void* workspace, size_t workspace_bytes,
                  int64_t count, int64_t* keys_out, float* vals_out, mkg_stream stream);
/* mkg_slab_emit of a sum hop with its normalisation (normalize_sparse3d(.., 0, "mass"),
 * drum.py:31-51) applied in the same pass: y_out the raw values, x_out = (y / d) * min(d, 1)
 * with d = row_sums[key row - row0] (fp32; the window's rows, complete and, across GPUs,
 * all-reduced), as mkg_mass_normalize; dropped (device int64) receives the number of results
 * that are zero or, when threshold > 0, below it. */
int mkg_slab_emit_normalized(const mkg_slab_window* win, void* store, const void* workspace, size_t workspace_bytes,
                             int64_t count, const float* row_sums, float threshold, int64_t* keys_out, float* y_out,
                             float* x_out, int64_t* dropped, mkg_stream stream);
/* Writes (mode 0), adds with a touched mark (mode 1) or raises to the maximum with a touched
 * mark (mode 2: max_sp_3d's max over rules with row_div = L) values at keys whose row is
 * (key / E) / row_div (row_div = L maps (b, l, e) to the [B, E] key b * E + e: sum_sp_3d,
 * fastlog_bridge.py:17-23).  mode | MKG_SLAB_SKIP_OUTSIDE skips the keys outside the window;
 * without it such a key (and always a negative one) sets MKG_DEV_BAD_KEY. */
int mkg_slab_put(const mkg_slab_window* win, void* store, const int64_t* keys, const float* vals, int64_t nnz,
                 int64_t row_div, int32_t mode, unsigned* dev_err, mkg_stream stream);
/* out[i] = the store's value at keys[i] (row (key / E) / row_div), cleared when clear & 1;
 * out may be NULL (clear only).  clear | MKG_SLAB_SKIP_OUTSIDE skips the keys outside the
 * window (their out[i] is left as it was). */
int mkg_slab_take(const mkg_slab_window* win, void* store, const int64_t* keys, int64_t nnz, int64_t row_div,
                  float* out, int32_t clear, unsigned* dev_err, mkg_stream stream);
/* Backward of mkg_slab_expand with the hop's output gradient held in the store (mode 0 puts):
 * grad_sp[i] += sum g m w[ch], grad_w[(b * L + l) * n + ch] += sum (g m) x, grad_edge[f] +=
 * g x w[ch] m dm/df -- replaces fastlog_backward_sparse3d_topk_cuda (fastlog.h:123-134,
 * fastlog.cu:3037-3109) with the edge-score gradient of fastlog_kernel.py:1032-1098.
 * grad_sp and grad_w are fp64 accumulators, grad_edge fp32; all are added to, not set. */
int mkg_slab_expand_backward(const int32_t* push_ptr, const mkg_adj_edge* push, const int64_t* keys,
                             const float* vals, int64_t nnz, const float* w, int64_t n, int32_t identity,
                             const mkg_slab_window* win, const void* store, const mkg_edge_factor* ef,
                             int64_t num_facts, double* grad_sp, double* grad_w, float* grad_edge, void* workspace,
                             size_t workspace_bytes, unsigned* dev_err, mkg_stream stream);
/* mkg_slab_expand_backward over ntiles destination tiles in one launch (as
 * mkg_slab_expand_tiles; the identity messages' gradient taken once, with tile 0). */
int mkg_slab_expand_backward_tiles(int32_t ntiles, const int32_t* const* push_ptrs, const mkg_adj_edge* const* pushes,
                                   const int64_t* keys, const float* vals, int64_t nnz, const float* w, int64_t n,
                                   int32_t identity, const mkg_slab_window* win, const void* store,
                                   const mkg_edge_factor* ef, int64_t num_facts, double* grad_sp, double* grad_w,
                                   float* grad_edge, void* workspace, size_t workspace_bytes, unsigned* dev_err,
                                   mkg_stream stream);
/* out[r] += sum of vals over the entries of row r (key / E - row0) in fp64; keys ascending.
 * The per-(b, l) sums of normalize_sparse3d and of its gradient (drum.py:31-51). */
int mkg_row_sums(const int64_t* keys, int64_t nnz, int64_t E, int64_t row0, int64_t nrows, const float* vals,
                 double* out, unsigned* dev_err, mkg_stream stream);
/* normalize_sparse3d(.., 0, "mass") (drum.py:31-51) on entries in any order: x = (y / d) *
 * min(d, 1) with d = row_sums[key / E - row0] (fp32).  dropped (device int64) receives the
 * number of results that are zero or, when threshold > 0, below it (the entries the loop
 * then drops). */
int mkg_mass_normalize(const int64_t* keys, const float* y, int64_t n, int64_t E, int64_t row0, int64_t nrows,
                       const float* row_sums, float threshold, float* x, int64_t* dropped, unsigned* dev_err,
                       mkg_stream stream);
/* Its gradient in two calls (a caller spanning several GPUs all-reduces `sums` in between):
 * mkg_mass_normalize_grad_sums adds sums[0][r] += gx * y / d and sums[1][r] += -(gx * min(d, 1)
 * * y) / d^2 over row r's entries (fp64, [2, nrows]; entries in any order); mkg_mass_normalize_grad writes
 * gy = gx * min(d, 1) / d + sums[1][r] + [d <= 1] sums[0][r] (zero where y is zero). */
int mkg_mass_normalize_grad_sums(const int64_t* keys, const float* y, const float* gx, int64_t n, int64_t E,
                                 int64_t row0, int64_t nrows, const float* row_sums, double* sums, unsigned* dev_err,
                                 mkg_stream stream);
/* mkg_mass_normalize_grad with gy written into a slab store at the keys' slots (the mode-0
 * mkg_slab_put before mkg_slab_expand_backward) instead of an array; every key must lie in
 * the window (else MKG_DEV_BAD_KEY). */
int mkg_mass_normalize_grad_put(const int64_t* keys, const float* y, const float* gx, int64_t n, int64_t E,
                                int64_t row0, int64_t nrows, const float* row_sums, const double* sums,
                                const mkg_slab_window* win, void* store, unsigned* dev_err, mkg_stream stream);
int mkg_mass_normalize_grad(const int64_t* keys, const float* y, const float* gx, int64_t n, int64_t E, int64_t row0,
                            int64_t nrows, const float* row_sums, const double* sums, float* gy, mkg_stream stream);
/* out[i] = (float) in[i]. */
int mkg_f64_to_f32(const double* in, int64_t n, float* out, mkg_stream stream);

/* ------------------------------------------------------------ bridge reducers */

/* Reduce-by-key of COO entries: replaces the torch coalescing behind sum_sparse3d_concat /
 * sum_sp_3d (src/fastlog_bridge.py:17-42) and the argsort / unique_consecutive /
 * scatter_reduce sequence of max_sp_3d / sparse3d_max (src/model_mmDRUM_kernel_sp.py:85-140,
 * 184-270).  keys (int64, >= 0, below 2^key_bits) with values; outputs in ascending key
 * order, one per distinct key: mode 0 the sum (fp64, rounded once), mode 1 the maximum, ties
 * to the earliest entry in input order.  out_keys / out_vals hold up to n entries;
 * count_out (device int64) receives the number written.  inverse [n] (may be NULL): output
 * index of each input entry; arg [n] (mode 1, may be NULL): the input entry that won each
 * output. */
/* sum_sp_3d / max_sp_3d (fastlog_bridge.py:17-23, model_mmDRUM_kernel_sp.py:184-236) on a
 * [B, L, E] state in entity-major order (keys (b * L + l) * E + e by ascending e, then row; the
 * order mkg_slab_emit writes): the rules of one (e, b) are adjacent, so each run is folded in
 * rule order (mode 0: fp32 sum, l ascending; mode 1: maximum) with no sort of the entries, and
 * one stable radix pass over the query puts the results in ascending b * E + e order.
 * out_keys / out_vals hold up to n results; count_out (device int64) receives their number;
 * out_pos [n] (may be NULL): each entry's result index.  Entries out of that order set
 * MKG_DEV_BAD_KEY. */
size_t mkg_rule_sum_workspace_bytes(int64_t n);
int mkg_rule_sum(const int64_t* keys, const float* vals, int64_t n, int64_t E, int64_t L, int64_t B, int32_t mode,
                 int64_t* out_keys, float* out_vals, int64_t* out_pos, int64_t* count_out, void* workspace,
                 size_t workspace_bytes, unsigned* dev_err, mkg_stream stream);

size_t mkg_reduce_by_key_workspace_bytes(int64_t n);
int mkg_reduce_by_key(const int64_t* keys, const float* vals, int64_t n, int32_t mode, int32_t key_bits,
                      int64_t* out_keys, float* out_vals, int64_t* count_out, int64_t* inverse, int64_t* arg,
                      void* workspace, size_t workspace_bytes, unsigned* dev_err, mkg_stream stream);

/* ------------------------------------------------------------ rule-weight producer */

typedef struct mkg_rule_params {
  int64_t n;   /* channels 2R + 1: rows of the relation embedding, outputs of the linear layer */
  int64_t H;   /* embedding size = LSTM input and hidden size (1 .. 112) */
  int64_t L;   /* rules: one bidirectional single-layer LSTM each */
  int64_t K;   /* hops: the LSTM sequence has K + 1 steps, the last output is dropped */
  int64_t U;   /* distinct target relations */
  int64_t B;   /* queries */
  float tau;   /* softmax temperature (tau_1) */
  int32_t reserved;
} mkg_rule_params;

/* Rule logits of the shared parametrisation: replaces SupplyGatedDRUM._shared_rule_logits
 * (drum.py:429-438) evaluated once per distinct target relation.  Parameters are fp32:
 * emb [n, H]; w_ih, w_hh [L, 2, 4H, H] (direction 0 = forward, 1 = reverse; gate rows i, f,
 * g, o as torch.nn.LSTM's weight_ih_l0 / weight_ih_l0_reverse); bias [L, 2, 4H] = b_ih + b_hh;
 * w_lin [n, 2H], b_lin [n]; rel_u [U] (int64, in [0, n)).  Writes logits_u [U, K, L, n]
 * (row u = the reference's output for a query of relation rel_u[u]) and keeps the LSTM
 * activations in `saved` (mkg_rule_saved_bytes) for the backward. */
size_t mkg_rule_saved_bytes(const mkg_rule_params* p);
int mkg_rule_logits_forward(const mkg_rule_params* p, const float* emb, const float* w_ih,
                            const float* w_hh, const float* bias, const float* w_lin,
                            const float* b_lin, const int64_t* rel_u, float* logits_u, void* saved,
                            size_t saved_bytes, unsigned* dev_err, mkg_stream stream);

/* Gradients of mkg_rule_logits_forward for grad_logits_u [U, K, L, n]: grad_emb [n, H],
 * grad_w_ih / grad_w_hh [L, 2, 4H, H], grad_bias [L, 2, 4H] (the gradient of b_ih and of
 * b_hh alike), grad_w_lin [n, 2H], grad_b_lin [n], all overwritten; sums in a fixed order
 * (no atomics). */
size_t mkg_rule_backward_workspace_bytes(const mkg_rule_params* p);
int mkg_rule_logits_backward(const mkg_rule_params* p, const float* emb, const float* w_ih,
                             const float* w_hh, const float* w_lin, const int64_t* rel_u,
                             const void* saved, size_t saved_bytes, const float* grad_logits_u,
                             float* grad_emb, float* grad_w_ih, float* grad_w_hh, float* grad_bias,
                             float* grad_w_lin, float* grad_b_lin, void* workspace,
                             size_t workspace_bytes, unsigned* dev_err, mkg_stream stream);

/* Per-hop rule weights of the hop loop (proof.py:569-571, decode_core.py:304):
 * w_hops[t, b, l, :] = softmax(logits_u[query_u[b], t, l, :] / tau), w_hops [K, B, L, n];
 * query_u [B] (int64, in [0, U)). */
int mkg_rule_softmax_forward(const mkg_rule_params* p, const float* logits_u, const int64_t* query_u,
                             float* w_hops, unsigned* dev_err, mkg_stream stream);

/* Gradient of mkg_rule_softmax_forward: grad_logits_u [U, K, L, n] (overwritten) from
 * w_hops and grad_w_hops [K, B, L, n]; the queries of relation u are
 * query_perm[query_ptr[u] .. query_ptr[u+1]) (int64 CSR), summed in that order. */
size_t mkg_rule_softmax_workspace_bytes(const mkg_rule_params* p);
int mkg_rule_softmax_backward(const mkg_rule_params* p, const float* w_hops, const float* grad_w_hops,
                              const int64_t* query_ptr, const int64_t* query_perm,
                              float* grad_logits_u, void* workspace, size_t workspace_bytes,
                              unsigned* dev_err, mkg_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* MINIKG_B200_H */
