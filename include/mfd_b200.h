/*
 * mfd_b200.h -- C ABI of the B200-native MFD verify step (libmfd_b200.so, sm_100a).
 *
 * Every entry point takes plain device pointers, element counts/strides and a cudaStream_t passed as
 * void*, launches on that stream without synchronising, allocates nothing (scratch comes from a caller
 * workspace) and returns an mfd_status; on failure mfd_last_error() describes the problem.  Host
 * bindings (mfd_b200/_lib.py, ctypes) raise RuntimeError on a nonzero status, as the reference's
 * TORCH_CHECKs do.  Each declaration names the reference interface it replaces
 * (hhhhhhy5/multi-future-drafting; "patch" = inference/sglang/patches/sglang-v0.5.22-mfd.patch).
 */
#ifndef MFD_B200_H
#define MFD_B200_H

#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

enum mfd_status {
    MFD_OK = 0,
    MFD_ERR_INVALID = 1,     /* bad argument: sizes, null pointers, dtype codes */
    MFD_ERR_UNSUPPORTED = 2, /* sizes beyond this build's limits */
    MFD_ERR_CUDA = 3,        /* a CUDA call failed */
    MFD_ERR_CAPACITY = 4     /* a device-side capacity check tripped (reported through a status word) */
};

enum mfd_dtype { MFD_F32 = 0, MFD_BF16 = 1, MFD_I32 = 2, MFD_I64 = 3 };

/* Thread-local message of the last failed call ("" if none). */
const char* mfd_last_error(void);
/* ABI version of this library. */
int mfd_abi_version(void);

/*
 * Logits step of tree construction: per row of x [rows, vocab] (row stride in elements), the top k
 * candidates ordered by value descending, equal values by lower index first, as
 *   top_logp[r, j] = x[r, ids[r, j]] - logsumexp(x[r, :])   (float32)
 * plus logz[r] (optional).  One pass over the logits.  k <= min(vocab, 256).
 * Replaces: inference/hf/ddtree.py:240-244 and 142-146 (torch.topk + torch.logsumexp),
 *           inference/hf/tree_logits.py:34-46 (row_logsumexp, top_candidates),
 *           patch:1472-1482 (row_logsumexp) and patch:1530-1545 (DDTreeDraftTopK.__call__ after its GEMM).
 * Scratch: mfd_topk_logz_workspace() bytes (no initialisation needed).  Tickets: `rows` uint32 words of a
 * buffer used only for tickets, zero before the first call; every kernel leaves its tickets zero again, so
 * one ticket buffer serves all calls that are stream-ordered with each other.
 */
size_t mfd_topk_logz_workspace(int64_t rows, int64_t vocab, int64_t k);
int mfd_topk_logz(const void* x, int x_dtype, int64_t rows, int64_t vocab, int64_t row_stride, int64_t k,
                  float* top_logp, void* top_ids, int ids_dtype, float* logz, void* workspace,
                  size_t workspace_bytes, unsigned int* tickets, int64_t tickets_len, void* stream);

/*
 * mfd_topk_logz for callers that may not allocate device memory at call time (a host whose memory pool owns
 * the whole GPU, a serving path where cudaMalloc's implicit synchronisation is not allowed, a plugin interface
 * that passes only inputs and outputs).  Same arguments, results and errors as mfd_topk_logz, without the
 * workspace and tickets: the scratch is one static device array in the library (4 MiB of partial records plus
 * tickets for 16384 rows; every GPU that loads the library holds it until the process exits).  Calls needing
 * more (mfd_topk_logz_workspace(rows, vocab, k) > 4 MiB, or rows > 16384) fail with MFD_ERR_UNSUPPORTED.
 * The first call on each device resolves the array's device address (make it before any stream capture; a
 * cudaDeviceReset after that first call is not supported, since the cached address would go stale).
 * All calls share the array: calls that may run at the same time on the GPU (other streams, other threads)
 * race; stream-ordered calls do not.  Allocates nothing.
 * Replaces: nothing in the reference (no counterpart; an allocation-free form of the entry point above).
 */
int mfd_topk_logz_static(const void* x, int x_dtype, int64_t rows, int64_t vocab, int64_t row_stride, int64_t k,
                         float* top_logp, void* top_ids, int ids_dtype, float* logz, void* stream);

/*
 * Exact best-first tree builders, batched, one request per CTA (bit-identical pop order).
 *   top_logp [bs, K, L, k] float32, top_ids [bs, K, L, k] int32/int64, log_prior [bs, K] (null = zeros).
 *   single = 1 (K must be 1): the DDTree heap, float64 key -logw, ties by the rank tuple;
 *   single = 0: the mixture heap, float32 key -(float(logw) + prior), ties by mode, parent, depth, rank,
 *   a prefix reached again by another mode reuses its node.
 * Outputs: tree [bs, 3, B+1] int64 (tokens, depths, parents; index 0 = root with token 0, depth 0,
 * parent -1; tail entries 0 / 0 / -1), counts [bs] int64; optional ancestor-or-self bitsets
 * anc_bits [bs, B+1, ceil((B+1)/64)] uint64 and/or dense visibility [bs, B+1, B+1] uint8.
 * status (optional device int) receives MFD_ERR_CAPACITY if a heap store overflows.
 * Limits: K <= 16, L <= 31, k <= 2047, B <= 511, K * (B + 1) <= 2048.
 * Replaces: patch:1375-1407 (build_trees / build_trees_cpu, SGLang);
 *           inference/hf/tree_build_ext.py:118-203 (build_single, build_mixture, finish);
 *           inference/hf/ddtree.py:161-211 and 259-314 (the Python heaps and the visibility loop).
 */
int mfd_build_trees(const float* top_logp, const void* top_ids, int ids_dtype, const float* log_prior, int64_t bs,
                    int64_t num_modes, int64_t depth_limit, int64_t topk, int64_t budget, int single, int64_t* tree,
                    int64_t* counts, uint64_t* anc_bits, uint8_t* visibility, int* status, void* stream);

/*
 * Target token per node and the verified-path walk in one launch.  logits: bf16 rows, row b*width + i
 * (row stride in elements).  temperature < 1e-5: argmax (first index of the maximum); otherwise one sample
 * per node by the reproducible rule documented in mfd_b200/csrc/accept.cu, with uniforms [bs*width].
 * The walk starts at node 0 and follows the child whose token equals the posterior (at most max_steps
 * edges; < 0 = unbounded).  Outputs (any may be null except posterior): posterior [bs*width];
 * accept_len [bs] (edges), commit_lens [bs] (= accept_len + 1), bonus [bs], out_tokens [bs, out_len]
 * (posterior along the path, then the bonus), accepted [bs, out_len] (node indices, -1 past the path),
 * new_seq_lens [bs] (= prefix + accept_len + 1), move_src/move_tgt [bs, out_len] (window slots),
 * hidden_index [bs, out_len] (= b*width + node).
 * Replaces: inference/hf/model/utils.py:28-35 (sample) + inference/hf/ddtree.py:368-382
 *           (follow_verified_tree) / tree_build_ext.py:70-83 (Tree.follow);
 *           patch:2986-3010 (_target_tokens) + patch:1844-1885 (ddtree_follow).
 * Scratch: mfd_accept_workspace(bs, width) bytes; tickets: mfd_accept_tickets(bs, width) zeroed words of a
 * ticket-only buffer (left zero again, as for mfd_topk_logz).
 */
size_t mfd_accept_workspace(int64_t bs, int64_t width);
int64_t mfd_accept_tickets(int64_t bs, int64_t width);
int mfd_accept(const void* logits, int64_t row_stride, int64_t vocab, int64_t bs, int64_t width,
               const int64_t* tokens, int64_t tokens_stride, const int64_t* parents, int64_t parents_stride,
               float temperature, const double* uniforms, int64_t max_steps, const int64_t* window,
               const int64_t* prefix_lens, int64_t out_len, int64_t* posterior, int32_t* accept_len,
               int32_t* commit_lens, int64_t* bonus, int64_t* out_tokens, int64_t* accepted, int64_t* new_seq_lens,
               int64_t* move_src, int64_t* move_tgt, int64_t* hidden_index, void* workspace,
               size_t workspace_bytes, unsigned int* tickets, int64_t tickets_len, void* stream);

/* Target token per row only (argmax or the reproducible sample).  Scratch: mfd_sample_tokens_workspace(rows)
 * bytes; tickets: rows + 1 zeroed words of a ticket-only buffer.
 * Replaces: inference/hf/model/utils.py:28-35 (sample); patch:2986-3010 (_target_tokens). */
size_t mfd_sample_tokens_workspace(int64_t rows);
int mfd_sample_tokens(const void* logits, int64_t row_stride, int64_t vocab, int64_t rows, float temperature,
                      const double* uniforms, int64_t* posterior, void* workspace, size_t workspace_bytes,
                      unsigned int* tickets, int64_t tickets_len, void* stream);

/* The walk alone, posterior given [bs, width].  Replaces: patch:1844-1885 (ddtree_follow). */
int mfd_follow(const int64_t* posterior, const int64_t* tokens, int64_t tokens_stride, const int64_t* parents,
               int64_t parents_stride, int64_t bs, int64_t width, int64_t max_steps, const int64_t* window,
               const int64_t* prefix_lens, int64_t out_len, int32_t* accept_len, int32_t* commit_lens,
               int64_t* bonus, int64_t* out_tokens, int64_t* accepted, int64_t* new_seq_lens, int64_t* move_src,
               int64_t* move_tgt, int64_t* hidden_index, void* stream);

/*
 * Verify inputs of a batch of trees: ids [bs, W] (root token at node 0), positions [bs, W] = prefix + depth,
 * and the flat int8 mask, request b's rows [W, prefix_b + W] at byte offset mask_offsets[b].
 * Replaces: patch:1625-1703 (_ddtree_verify_inputs_kernel / ddtree_verify_inputs).
 */
int mfd_verify_inputs(const int64_t* root_tokens, const int64_t* prefix_lens, const int64_t* tokens,
                      const int64_t* depths, const int64_t* parents, int64_t tree_stride, const int64_t* mask_offsets,
                      int64_t bs, int64_t width, int64_t max_depth, int64_t* ids_out, int64_t* positions_out,
                      int8_t* mask_out, void* stream);

/*
 * HF verify inputs of one tree, in the caller's buffers: ids[0] = *root_token, ids[i] = tokens[i]; positions[i] =
 * start + depths[i] (i < n, node 0 the root); the tree block of the additive mask, mask[i, past_length + j] = 0
 * where vis[i, j] != 0 else the bits min_bits (i, j < n); the previous round's block mask[i, prev_start + j]
 * (i, j < prev_length) reset to 0 outside the new block; vis_out[i, j] = vis[i, j] (bool).  root_token, tokens,
 * depths (int64), vis ([n, vis_stride] uint8) on the device.  mask: [mask_rows, mask_cols] elements of
 * mask_elem_bytes (2: bf16 / fp16, 4: fp32) with row stride mask_row_stride elements; both blocks must lie inside.
 * Replaces: inference/hf/ddtree.py:317-357 (compile_ddtree_tree: its host-to-device copies of ids, depths and
 * visibility and the fill / masked_fill of the mask block).
 */
int mfd_compile_tree(const int64_t* root_token, const int64_t* tokens, const int64_t* depths, int64_t n,
                     const uint8_t* vis, int64_t vis_stride, int64_t start, int64_t past_length, int64_t prev_start,
                     int64_t prev_length, int64_t* ids_out, int64_t* positions_out, void* mask,
                     int64_t mask_elem_bytes, int64_t mask_row_stride, int64_t mask_rows, int64_t mask_cols,
                     uint32_t min_bits, bool* vis_out, int64_t vis_out_stride, void* stream);

/*
 * Tree-masked GQA verify attention on the tcgen05 tensor cores.  q, out [bs, n, H, 128] bf16 (strides in elements,
 * multiples of 8, last dim contiguous); k, v [bs, Hkv, max_keys, 128] bf16 holding each request's prefix keys
 * followed by its n tree keys (keys at or past max_keys are never read); prefix_lens [bs] int32 on the device (or
 * null: every request uses prefix_len); anc_bits [bs, n, words] ancestor-or-self bitsets (mfd_build_trees).  Row i
 * sees all prefix keys and the tree keys of its ancestors and itself.  The keys are split into `splits` ranges;
 * the last range to finish merges them by log-sum-exp.  H / Hkv must divide 128.
 * Replaces: the target's SDPA call with the compile_ddtree_tree mask (inference/hf/ddtree.py:352-356,
 *           598-605); SGLang's flashinfer custom-mask prefill (patch:86-142, 558-592); with a block-diagonal
 *           visibility, the drafter's mode_block_attention (inference/hf/mode_attention.py:120-150).
 * Workspace: mfd_tree_attention_workspace(bs, n, H, Hkv, splits) bytes, zeroed before its first use; its first
 * int32 (at the 256-byte aligned base) is a sticky device status: 1 once a bounded wait in the kernel gave up, 2 if
 * a CTA's shared-memory base was misaligned beyond the slack it reserves (that CTA did no work); the caller reads
 * and clears it.  Tickets (splits > 1): mfd_tree_attention_tickets(bs, n, H, Hkv) zeroed words of a ticket-only
 * buffer, left zero again (as for mfd_topk_logz); the workspace itself may be reused with any sizes.
 */
size_t mfd_tree_attention_workspace(int64_t bs, int64_t n, int64_t num_heads, int64_t num_kv_heads, int64_t splits);
int64_t mfd_tree_attention_tickets(int64_t bs, int64_t n, int64_t num_heads, int64_t num_kv_heads);
int mfd_tree_attention(const void* q, int64_t sq_b, int64_t sq_n, int64_t sq_h, const void* k, int64_t sk_b,
                       int64_t sk_h, int64_t sk_s, const void* v, int64_t sv_b, int64_t sv_h, int64_t sv_s,
                       int64_t max_keys, const int32_t* prefix_lens, int64_t prefix_len, const uint64_t* anc_bits,
                       int64_t anc_words, int64_t bs, int64_t n, int64_t num_heads, int64_t num_kv_heads,
                       int64_t head_dim, float scale, int64_t splits, void* out, int64_t so_b, int64_t so_n,
                       int64_t so_h, void* workspace, size_t workspace_bytes, unsigned int* tickets,
                       int64_t tickets_len, void* stream);

/*
 * Paged multi-mode draft attention of a serving batch: bs requests, each with num_modes blocks of block_size
 * queries side by side (n = num_modes * block_size rows per request, mode-major).  Query i of request b attends to
 * the request's context -- rows req_to_token[req_pool_indices[b] * r2t_stride + j] of k_cache / v_cache for
 * j < ctx_lens[b] (clamped to [0, r2t_cols]; req_pool_indices clamped to [0, r2t_rows)) -- and to the block keys
 * of its own mode, rows b n + j of k_new / v_new, as block_bits says ([n, bits_words] bitsets, one set for every
 * request: row i sees block key j when bit j of row i is set).  q, out [bs n, H, 128] (token stride sq_t / so_t,
 * head stride sq_h / so_h); k_new, v_new [bs n, Hkv, 128] and k_cache, v_cache [num_slots, Hkv, 128] bf16 with
 * the KV heads of a token contiguous (head stride 128, token strides multiples of 8, K and V alike);
 * req_to_token int32, req_pool_indices and ctx_lens int64, all on the device.  Slot ids are clamped to
 * [0, num_slots).  The grid depends only on the sizes and `splits`; the lengths are read on the device.
 * Workspace and tickets: as for mfd_tree_attention with (bs, n, H, Hkv, splits).
 * Replaces: SGLang's paged_mode_block_attention (patch:897-962) and its Triton split / merge / fused kernels
 *           (patch:627-880), called by PagedModeAttention (patch:991-1026).
 */
int mfd_paged_mode_attention(const void* q, int64_t sq_t, int64_t sq_h, const void* k_new, int64_t skn_t,
                             int64_t skn_h, const void* v_new, int64_t svn_t, int64_t svn_h, const void* k_cache,
                             int64_t skc_t, int64_t skc_h, const void* v_cache, int64_t svc_t, int64_t svc_h,
                             int64_t num_slots, const int32_t* req_to_token, int64_t r2t_rows, int64_t r2t_cols,
                             int64_t r2t_stride, const int64_t* req_pool_indices, const int64_t* ctx_lens,
                             const uint64_t* block_bits, int64_t bits_words, int64_t bs, int64_t num_modes,
                             int64_t block_size, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                             float scale, int64_t splits, void* out, int64_t so_t, int64_t so_h, void* workspace,
                             size_t workspace_bytes, unsigned int* tickets, int64_t tickets_len, void* stream);

/*
 * Tree verification of one gated-delta-rule layer from the committed state S0 (fla layout, o = S^T q):
 *   u_i + sum_{j strict ancestor of i} beta_i e^{G_i-G_j} (k_i.k_j) u_j = beta_i (v_i - e^{G_i} S0^T k_i)
 *   o_i = e^{G_i} S0^T q_i + sum_{j ancestor of i or i} e^{G_i-G_j} (q_i.k_j) u_j
 *   states_i = e^{G_i} S0 + sum_{j ancestor of i or i} e^{G_i-G_j} k_j u_j^T      (only if states != null)
 * q, k [n, HK, Dk] bf16 (node strides sq, sk; q already l2-normalised and scaled, k l2-normalised); v [n, H, Dv]
 * bf16 (node stride sv); g_cum, beta [n, H] float32 (node strides sg, sb; g_cum = log decay summed along the root
 * path); s0 [H, Dk, Dv] float32; anc [n, n] int8 (row stride sa), row i = ancestors of i and i, nodes in
 * topological order.  Value head h reads key head h / (H / HK).  Outputs u, o [n, H, Dv] float32 and, if
 * states != null, states [n, H, Dk, Dv] float32.  status (optional, device int): 0; 1 when anc is not the
 * ancestor matrix of a topologically ordered tree; MFD_ERR_CAPACITY when the tree's ancestor pairs (the sum over
 * nodes of depth + 1) exceed what the kernel holds at this n (any tree of up to 128 nodes fits; 257 nodes: 6.7
 * thousand pairs); 3 if a bounded wait gave up.  Outputs are unspecified unless the status is 0.
 * Limits: n <= 384, Dk <= 128 and a multiple of 8, Dv a multiple of 4 (<= 128 when states are written).
 * The contractions run on the tcgen05 tensor cores (S0^T k, S0^T q and the Gram products per 128-node tile; one
 * path contraction per node and head for the states).
 * Replaces: inference/hf/tree_gdn_kernel.py:153-171 (tree_gdn: _tree_kkt, fla solve_tril, _tree_u), and the
 *           state formula of inference/hf/qwen35_tree.py:134-137 evaluated for every node.
 */
int mfd_tree_gdn(const void* q, int64_t sq, const void* k, int64_t sk, const void* v, int64_t sv,
                 const float* g_cum, int64_t sg, const float* beta, int64_t sb, const float* s0, const int8_t* anc,
                 int64_t sa, int64_t n, int64_t num_heads, int64_t num_k_heads, int64_t dk, int64_t dv, float* u,
                 float* o, float* states, int* status, void* stream);

/*
 * Gates of a Gated-DeltaNet layer over a tree, per node i and value head h: beta = sigmoid(b[i, h]),
 * g = -exp(A_log[h]) * softplus(a[i, h] + dt_bias[h]), and G[i, h] = the sum of g over the root path of i (i
 * included).  a, b [n, H] (row strides sa, sb in elements; ab_dtype MFD_BF16 or MFD_F32), A_log and dt_bias [H]
 * float32, parents [n] int64 (parents[i] < i, -1 for a root) on the device; outputs beta, G [n, H] float32.
 * n <= 2048.  status (optional device int) receives MFD_ERR_INVALID for a parent that is not an earlier node
 * (that node is treated as a root).
 * Replaces: inference/hf/qwen35_tree.py:77-79 (sigmoid, softplus decay, G = anc_f @ g).
 */
int mfd_tree_gates(const void* a, int64_t sa, const void* b, int64_t sb, int ab_dtype, const float* a_log,
                   const float* dt_bias, const int64_t* parents, int64_t n, int64_t num_heads, float* beta, float* G,
                   int* status, void* stream);

/*
 * Inputs of mfd_tree_gdn from the pre-convolution projections: per node i and channel c,
 *   y = bf16(silu(sum_t w[c][t] * X[conv_index[i][t]][c]))  with X = [conv_state^T ; x] (window oldest first),
 * then q, k heads l2-normalised (y / sqrt(sum y^2 + 1e-6)), q times scale.  x [n, conv_dim] bf16 with
 * conv_dim = (2 HK + H) D (channels: q heads, k heads, v heads); conv_state, conv_w [conv_dim, kernel] bf16;
 * conv_index [n, kernel] int32.  Outputs q, k [n, HK, D], v [n, H, D] bf16 (contiguous).  D <= 128.
 * Replaces: inference/hf/tree_gdn_kernel.py:135-150 (tree_prep, the _tree_prep kernel at 27-56).
 */
int mfd_tree_prep(const void* x, const void* conv_state, const int32_t* conv_index, const void* conv_w, int64_t n,
                  int64_t conv_dim, int64_t kernel, int64_t num_k_heads, int64_t num_heads, int64_t head_dim,
                  float scale, void* q, void* k, void* v, void* stream);

/*
 * Commit step, KV moves in a token-major pool (SGLang).  buffers: a device array of num_buffers base addresses
 * (every layer's K and V buffer), each holding slots of slot_bytes (a multiple of 8).  base_align: an alignment in
 * bytes (a multiple of 8) that every buffer base has; the kernel moves 16-byte units only when slot_bytes and
 * base_align are multiples of 16, else 8-byte units, so a base must be at least 8-byte aligned.  For request b and
 * i < width, slot move_src[b, i] moves to move_tgt[b, i] in every buffer when the two differ; every source is read
 * before any store (a path slot can be another move's target).  move_src, move_tgt [bs, width] int64 on the device
 * (width <= 1024); negative ids are no-ops.  pool_slots > 0 bounds the slot ids: a move whose source or target is
 * >= pool_slots is skipped and status (optional device int) receives MFD_ERR_INVALID; 0 leaves them unchecked.
 * One launch for all buffers.
 * Replaces: patch:1769-1841 (DDTreeKVCompactor / _ddtree_compact_kv_kernel).
 */
int mfd_commit_kv_moves(const uint64_t* buffers, int64_t num_buffers, int64_t slot_bytes, int64_t base_align,
                        const int64_t* move_src, const int64_t* move_tgt, int64_t bs, int64_t width,
                        int64_t pool_slots, int* status, void* stream);

/*
 * Commit step, HF cache compaction.  buffers: a device array of num_buffers base addresses of cache tensors viewed
 * as [outer, rows, row_bytes] (outer_stride and row_stride in bytes, multiples of 8).  base_align: an alignment in
 * bytes (a multiple of 8) that every buffer base has; 16-byte units are used only when it, row_bytes and both
 * strides are multiples of 16.  Row past_length + keep[i] moves to past_length + i for i < keep_count in every
 * buffer and outer index; nothing happens when the appended window rows - past_length is empty, or keep_count is
 * 0 or the whole window (as the reference returns early).  keep [keep_count] int64 on the device
 * (keep_count <= 1024); status (optional device int) receives MFD_ERR_INVALID for a keep index outside the window
 * (that move is skipped).
 * Replaces: inference/hf/ddtree.py:33-61 (compact_tail_inplace), 385-403 (_compact_appended_window), applied by
 *           406-436 (compact_dynamic_cache) to every layer's keys and values.
 */
int mfd_compact_tail(const uint64_t* buffers, int64_t num_buffers, int64_t outer, int64_t outer_stride, int64_t rows,
                     int64_t row_stride, int64_t row_bytes, int64_t base_align, int64_t past_length,
                     const int64_t* keep, int64_t keep_count, int* status, void* stream);

/*
 * Commit step of the Gated-DeltaNet layers: every layer's recurrent state (in place) becomes the state at the
 * deepest accepted node a = path[path_len - 1]:
 *   S_a = e^{G_a} S0 + sum_{j in path} e^{G_a - G_j} k_j u_j^T   (value head h reads key head h / (H / HK)).
 * Per layer (device arrays of base addresses): states [H, Dk, Dv] (state_dtype MFD_F32 or MFD_BF16), u [n, H, Dv]
 * float32, k [n, HK, Dk] bf16, g_cum [n, H] float32 (the cumulative decays G), all contiguous.  path [path_len]
 * int64 on the device (1..128 nodes).  Dv a multiple of 4, <= 256; the state bases 16-byte aligned.
 * Replaces: inference/hf/qwen35_tree.py:122-137 (commit, the state part, over the stacked layers).
 */
int mfd_gdn_commit(const uint64_t* states, int state_dtype, const uint64_t* u, const uint64_t* k, const uint64_t* g_cum,
                   int64_t layers, const int64_t* path, int64_t path_len, int64_t n, int64_t num_heads,
                   int64_t num_k_heads, int64_t dk, int64_t dv, void* stream);

/*
 * Commit step of the causal-conv windows: per layer and channel c, column t of conv_states [conv_dim, kernel]
 * becomes window[t] < kernel ? the old column window[t] : x[window[t] - kernel][c] (x [n, conv_dim], same
 * element type, elem_bytes 2 or 4), the whole window read before it is written.  window [kernel] int32 on the
 * device (the accepted node's window, TreeContext.conv_index); kernel <= 8.
 * Replaces: inference/hf/qwen35_tree.py:138-146 (commit, the conv part).
 */
int mfd_conv_commit(const uint64_t* conv_states, const uint64_t* x, int64_t elem_bytes, int64_t layers,
                    int64_t conv_dim, int64_t kernel, const int32_t* window, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MFD_B200_H */
