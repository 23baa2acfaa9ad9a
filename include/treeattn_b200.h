/* treeattn_b200 - C ABI of the B200 (sm_100a) segment-tree sparse-attention kernels.
 *
 * Conventions (every entry point):
 *   - All pointers are device pointers owned by the caller; the library allocates nothing on these paths.
 *   - Strides are in ELEMENTS; the innermost (head-dim) stride is 1. Rows read with 16-byte vector loads
 *     or bulk copies must start 16-byte aligned (checked; violations return TA_ERR_ARG).
 *   - dtype codes: 0 = float32, 1 = bfloat16, 2 = float16.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Work is only enqueued; nothing synchronizes.
 *   - Return value: 0 on success, TA_ERR_ARG for rejected arguments, TA_ERR_CUDA for a launch failure.
 *     ta_last_error() then describes the failure (thread-local string). There is no fallback path.
 *   - Kernels that detect a bad position/index at run time, or a bounded wait that gave up, record it in a
 *     device-side error record read (and cleared) by ta_device_error().
 *
 * Tree levels ("nodes"): per (b, h) the levels L0..Lm are packed back to back, level l holding cap >> l fp32
 * rows of dh values (node m covers positions [m*2^l, (m+1)*2^l)); n_sb / n_sh are the strides (in floats)
 * between batch rows / heads. ta_level_nodes() gives the per-(b, h) node count.
 */
#ifndef TREEATTN_B200_H
#define TREEATTN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TA_OK 0
#define TA_ERR_ARG 1
#define TA_ERR_CUDA 2

#define TA_F32 0
#define TA_BF16 1
#define TA_F16 2

/* Library version (major*10000 + minor*100 + patch). */
int ta_version(void);

/* Description of the last failure on this thread ("" if none). */
const char* ta_last_error(void);

/* Copy the device-side error record {code, kernel, a, b} of the current device into out4 and clear it.
 * Synchronizes the device. code 0 = no error, 1 = bounded wait gave up, 2 = position out of range,
 * 3 = index out of range. */
int ta_device_error(int* out4);

/* No counterpart in the reference: a test of the kernels' bounded waits. One CTA waits on an mbarrier that no
 * thread arrives at; after limit_ns (1 us .. 10 s) it gives up, records code 1 (bounded wait gave up) with
 * kernel id 13 in the device-side error record and ends normally, so that the context stays usable. The
 * library's own waits give up the same way, after 2 s. */
int ta_wait_probe(int64_t limit_ns, void* stream);

/* Nodes per (b, h) for a capacity and level range: sum over l in [L0, Lm] of cap >> l. */
int64_t ta_level_nodes(int cap, int L0, int Lm);

/* Replaces seg.level_sums (seg.py:26-41), fastseg.level_sums_min (fastseg.py:238-251) and the bulk
 * SegState.fill (engine.py:57-71): node sums of levels L0..Lm from keys k (B, H, T_len, dh), complete nodes
 * only (m < T_len >> l). zero_sink != 0 counts the key at position 0 as 0 (what select_seg and SegState do,
 * seg.py:128-130, engine.py:62). fp32, reference pair order (bit-exact). */
int ta_build_levels(const void* k, int dtype, int B, int H, int T_len, int dh, int64_t k_sb, int64_t k_sh,
                    int64_t k_st, int cap, int L0, int Lm, int zero_sink, float* nodes, int64_t n_sb, int64_t n_sh,
                    void* stream);

/* The mean-log gate's statistic tree (seg.py:26-41 and fastseg.py:238-251 with cfg.gate, engine.py:47-54):
 * arguments and layout as ta_build_levels; the leaf-level nodes sum log(|k| + 1e-6) of the (sink-zeroed) keys
 * instead of the keys, in the same adjacent-pair order. */
int ta_build_log_levels(const void* k, int dtype, int B, int H, int T_len, int dh, int64_t k_sb, int64_t k_sh,
                        int64_t k_st, int cap, int L0, int Lm, int zero_sink, float* nodes, int64_t n_sb,
                        int64_t n_sh, void* stream);

/* Replaces seg.gate_apply (seg.py:16-23) over whole trees (fastseg.level_sums_min, fastseg.py:238-251): for every
 * complete node (m < T_len >> l) of levels gate_min..Lm, out = raw * [ml >= q-quantile of ml] * dh / kept with
 * ml = lg / 2^l (torch.quantile's interpolation); levels below gate_min are copied. raw, lg, out share the packed
 * layout of ta_build_levels (strides n_sb, n_sh). dh 16, 32, 64 or 128. */
int ta_gate_levels(const float* raw, const float* lg, float* out, int B, int H, int dh, int T_len, int64_t n_sb,
                   int64_t n_sh, int cap, int L0, int Lm, float gate_q, int gate_min, void* stream);

/* Decoding with the gate (engine.py:33-37 getU, 41-55 add): after ta_append / ta_decode_step appended position
 * pos[b], forms the log-magnitude nodes completed by pos[b] (leaf block read from the key cache kc, right-spine
 * ancestors) and the gated copies of every node formed at pos[b]. */
int ta_gate_append(const void* kc, int dtype, int B, int H, int dh, int64_t c_sb, int64_t c_sh, int64_t c_st,
                   const float* raw, float* lg, float* out, int64_t n_sb, int64_t n_sh, int cap, int L0, int Lm,
                   const int32_t* pos, float gate_q, int gate_min, void* stream);

/* Replaces seg.tree_pass (seg.py:44-70) / fastseg.tree_pass_fast (fastseg.py:254-271) on the tree of leaf
 * blocks of 2^L0 tokens: per query (b, h, n) at position tq[b*tq_sb + n*tq_st], the best wmax leaves, best
 * first. Outputs (B, H, Nq, wl) contiguous: ids (int64, invalid slots 0), vld (uint8), sct (fp32 scores
 * q.S_L0 / 2^L0, -inf when invalid; may be NULL). q may be float32, bfloat16 or float16 (q_dtype). */
int ta_select(const void* q, int q_dtype, int B, int H, int Nq, int dh, int64_t q_sb, int64_t q_sh, int64_t q_st,
              const int64_t* tq, int64_t tq_sb, int64_t tq_st, const float* nodes, int64_t n_sb, int64_t n_sh,
              int cap, int L0, int Lm, int wmax, int wl, int64_t* ids, uint8_t* vld, float* sct, void* stream);

/* Replaces seg.finish + seg.leaves_to_pos (seg.py:106-119) for Q queries: n_tree from the budget lhat and the
 * neighbour count nL (NULL = 0); leaf ids -> positions (tree_pos[q, j*wl + i] = ids[q, i]*leaf + j, -1 when
 * invalid); neighbour leaves likewise (nid/match NULL = no matches). tree_pos / nb_pos may be NULL when only
 * n_tree and nb_leaves are wanted. */
int ta_finish(const int64_t* ids, const uint8_t* vld, const int64_t* nid, const uint8_t* match, const int64_t* nL,
              const int64_t* lhat, int64_t Q, int wl, int nbw, int leaf, int wmax, int64_t* tree_pos,
              int64_t* nb_pos, int64_t* n_tree, int64_t* nb_leaves, void* stream);

/* Replaces the key assembly + dedupe_fast + sparse_attn of SegAttention.sparse_attend (fastseg.py:367-383)
 * and DynAttention.sparse_attend (attention_dyn.py:345-366): per query, exact softmax attention (scale,
 * fp32 accumulation) over the first n_tree valid leaves of ids/vld (each 2^L0 positions), the sink and the
 * window [t-Lw+1, t], every position once. o has q's dtype; lse (natural log) and nkeys may be NULL.
 * n_tree NULL -> ntree_const for every query. */
int ta_seg_attn(const void* q, const void* k, const void* v, int dtype, int B, int H, int Nq, int dh,
                int64_t q_sb, int64_t q_sh, int64_t q_st, int64_t k_sb, int64_t k_sh, int64_t k_st,
                int64_t v_sb, int64_t v_sh, int64_t v_st, int T_kv, const int64_t* tq, int64_t tq_sb,
                int64_t tq_st, const int64_t* ids, const uint8_t* vld, int wl, const int64_t* n_tree,
                int ntree_const, int leaf, int Lw, float scale, void* o, int64_t o_sb, int64_t o_sh, int64_t o_st,
                float* lse, int32_t* nkeys, void* stream);

/* Same computation and arguments as ta_seg_attn (fastseg.py:367-383: static keys, dedupe_fast, _attn_fwd), on
 * the tensor cores for whole sequences (prefill): 128 queries of one (b, h) per CTA stream the union of their
 * key sets in 64-key tiles (tcgen05.mma into tensor memory, TMA loads), each query masked to its own
 * deduplicated keys. bf16 / f16, dh 64 or 128, leaf >= 2, at most 1024 leaf blocks per sequence (T_kv / leaf); queries of
 * a 128-tile should be close in position (the window union is streamed). */
int ta_prefill_attn(const void* q, const void* k, const void* v, int dtype, int B, int H, int Nq, int dh,
                    int64_t q_sb, int64_t q_sh, int64_t q_st, int64_t k_sb, int64_t k_sh, int64_t k_st,
                    int64_t v_sb, int64_t v_sh, int64_t v_st, int T_kv, const int64_t* tq, int64_t tq_sb,
                    int64_t tq_st, const int64_t* ids, const uint8_t* vld, int wl, const int64_t* n_tree,
                    int ntree_const, int leaf, int Lw, float scale, void* o, int64_t o_sb, int64_t o_sh,
                    int64_t o_st, float* lse, int32_t* nkeys, void* stream);

/* Replaces fastseg.sparse_attn forward (fastseg.py:173-177, _attn_fwd 49-78): cand (B, H, T, Kc) key
 * positions (int32 if cand64 == 0, else int64), -1 = unused. o (B, H, T, dh) in q's dtype, lse may be NULL. */
int ta_sparse_attn(const void* q, const void* k, const void* v, int dtype, int B, int H, int T, int dh,
                   int64_t q_sb, int64_t q_sh, int64_t q_st, int64_t k_sb, int64_t k_sh, int64_t k_st,
                   int64_t v_sb, int64_t v_sh, int64_t v_st, int T_kv, const void* cand, int cand64, int Kc,
                   float scale, void* o, int64_t o_sb, int64_t o_sh, int64_t o_st, float* lse, void* stream);

/* Replaces seg.neighbor_pass (seg.py:73-103) / fastseg.neighbor_pass_fast (fastseg.py:274-299) on leaf blocks of
 * 2^L0 tokens: query (b, h, n) at position tq[b*tq_sb + n*tq_st] re-scores the nb_store best leaves stored by each
 * of the nb_window previous positions (st_leaf / st_score / st_ok (B, H, T_st, nb_store) contiguous, indexed by
 * position) against the level-L0 node rows leaf_nodes (row m of (b, h) at + b*n_sb + h*n_sh + m*dh, n_leaf rows)
 * and matches those it scores at least base - nb_rho |base|, scanning no deeper than nb_cap_min +
 * round((nb_window - nb_cap_min) * match rate over the first nb_probe positions). neighbors == 0 reproduces
 * cfg.neighbors=False (no matches). Outputs (B, H, Nq, nb_window*nb_store) contiguous: nid (the stored ids), match;
 * nL (B, H, Nq) = distinct matched leaves. nb_window * nb_store <= 32. */
int ta_neighbor_pass(const void* q, int q_dtype, int B, int H, int Nq, int dh, int64_t q_sb, int64_t q_sh,
                     int64_t q_st, const int64_t* tq, int64_t tq_sb, int64_t tq_st, const float* leaf_nodes,
                     int64_t n_sb, int64_t n_sh, int n_leaf, int L0, const int64_t* st_leaf, const float* st_score,
                     const uint8_t* st_ok, int T_st, int nb_window, int nb_store, float nb_rho, int nb_probe,
                     int nb_cap_min, int neighbors, int64_t* nid, uint8_t* match, int64_t* nL, void* stream);

/* Replaces dyntree.LaneTree.search (dyntree.py:108-127): beam descent for one query per lane over a dynamic
 * content tree whose nodes hold key sums and counts. q (P, dh) fp32; sums (P, 2^(D+1) - 1, dh) fp32 and cnt
 * (P, 2^(D+1) - 1) int32 packed level by level (level l at rows 2^l - 1 .. 2^(l+1) - 2, l = 0..D). A child is valid
 * when its parent is and its count is positive and scores q . sum / count; per level the best min(wmax, 2 * width)
 * are kept. Outputs (P, wl) best first: node ids of level D (0 when invalid), validity, scores (-inf when invalid;
 * sct may be NULL). */
int ta_lane_search(const float* q, const float* sums, const int32_t* cnt, int P, int D, int dh, int wmax, int wl,
                   int64_t* ids, uint8_t* vld, float* sct, void* stream);

/* Replaces the 2-means splits of the dyntree.LaneTree build (dyntree.py:6-31 masked_two_means_order and 54-73) and,
 * with all slots valid, forest.build_forest's content sort (forest.py:13-33 two_means_order, 59-67). Lane p orders
 * C slots (a power of two, 4..16384); slot s holds key row s of the lane's key array, fp32 (C, dh) at
 * keys + (p / key_lane_div) * key_stride, and is valid when first <= s < n[p]. For every level lvl < `levels` the
 * valid keys of each group of C >> lvl slots are sorted by their projection on the difference of two 2-means
 * centres (iters rounds) and dealt to the group's halves, ceil(count / 2) to the left. Output perm (P, C) int32
 * (the key row in every slot) and valid (P, C) uint8; perm_tmp / valid_tmp are scratch of the same sizes. */
int ta_lane_order(const float* keys, int64_t key_lane_div, int64_t key_stride, const int64_t* n, int first, int P,
                  int C, int dh, int iters, int levels, int32_t* perm, uint8_t* valid, int32_t* perm_tmp,
                  uint8_t* valid_tmp, void* stream);

/* No counterpart in the reference: ta_lane_order for callers that cannot allocate device memory - for instance a
 * host program that reserved the GPU's memory up front for its own pool and hands the library only views into it,
 * so that a cudaMalloc would fail or break its accounting. The build's second slot-order buffer is a static array
 * inside the library (2^21 slots: P * C at most, 10 MiB held on every GPU that loads the library); the call itself
 * calls no allocator. Larger P * C is rejected with TA_ERR_ARG. The array's device address belongs to one CUDA
 * context: each call made outside stream capture looks it up with the calling thread's current context (so a
 * cudaDeviceReset or another context made current in between is followed), and records it for that context; a call
 * whose stream is capturing reuses the address recorded for the current context, so the first call in a context
 * must come before any stream capture (otherwise TA_ERR_ARG). All calls share
 * the array (it is fully rewritten by each call, nothing needs clearing): calls that overlap on the GPU race, so
 * order them (one stream, or events). Same arguments and results as ta_lane_order otherwise. */
int ta_lane_order_noalloc(const float* keys, int64_t key_lane_div, int64_t key_stride, const int64_t* n, int first,
                          int P, int C, int dh, int iters, int levels, int32_t* perm, uint8_t* valid, void* stream);

/* Completes a dyntree.LaneTree build (dyntree.py:74-80): from the ordered slots of ta_lane_order, the group slots
 * slot (P, C/2, 2) int32 (key position, -1 = empty) and the node sums (P, C - 1, dh) fp32 / counts (P, C - 1) int32
 * packed level by level (level l at rows 2^l - 1 .. 2^(l+1) - 2), formed bottom-up in adjacent pairs. */
int ta_lane_sums(const float* keys, int64_t key_lane_div, int64_t key_stride, const int32_t* perm,
                 const uint8_t* valid, int P, int C, int dh, float* sums, int32_t* cnt, int32_t* slot, void* stream);

/* Replaces dyntree.LaneTree.insert (dyntree.py:83-106): key kv[p] (fp32, dh) at position kpos[p] joins lane p's
 * tree where active[p]: added to the root and, level by level, to the child whose mean scores higher against it
 * (kv . sum / count; -1e9 when empty, -inf when full; ties left), then to the first free slot of its group. */
int ta_lane_insert(const float* kv, const int64_t* kpos, const uint8_t* active, int P, int C, int dh, float* sums,
                   int32_t* cnt, int32_t* slot, void* stream);

/* Replaces dyntree.select_keys (dyntree.py:150-243) after the build: lane p = (b H + h) (T / chunk) + l holds the
 * tree of the keys [1, l chunk) of (b, h) (ta_lane_order + ta_lane_sums with key_lane_div = T / chunk) and walks
 * the tokens t = l chunk .. (l + 1) chunk - 1 in order: neighbour rescoring of the nb_store best groups stored by
 * the previous nb_window tokens of the lane (q . sum / count >= base - rho |base|, scan depth capped by the probe
 * rate), the beam descent (as ta_lane_search), the tree budget from lhat, and the insertion of the token's key
 * (t >= 1). q, k (B, H, T, dh) fp32; lhat (B, H, T) int64. Outputs tree_pos (B, H, T, 2 wl), leaf_ok (B, H, T, wl),
 * nb_pos (B, H, T, 2 nb_window nb_store) int64 positions (-1 = none), n_tree, nb_leaves (B, H, T) int64;
 * wl = min(wmax, T / 2). The trees are updated in place. */
int ta_lane_select(const float* q, const float* k, const int64_t* lhat, int B, int H, int T, int dh, int chunk,
                   int wmax, int nb_window, int nb_store, int nb_probe, int nb_cap_min, float nb_rho, int neighbors,
                   float* sums, int32_t* cnt, int32_t* slot, int64_t* tree_pos, uint8_t* leaf_ok, int64_t* nb_pos,
                   int64_t* n_tree, int64_t* nb_leaves, void* stream);

/* Replaces the node sums of forest.build_forest (forest.py:68-75) and forest.soft_gate (forest.py:36-44): per block
 * p of B keys (rows p B .. p B + B - 1 of k, dtype code `dtype`, dh wide; with zero_sink the key at position 0 of
 * every (b, h) - the first row of blocks p % nb == 0 - counts as 0), ranks ordered by perm (P, B) int32 (from
 * ta_lane_order with every slot valid), level l = 0..depth (depth = log2(B / 2)) holds 2^l nodes summing B / 2^l
 * keys each; out[l] (P 2^l, dh) in k's dtype. gate != 0 applies the soft mean-log gate (gate_q, gate_temp). */
int ta_forest_levels(const void* k, int dtype, int P, int B, int dh, int depth, int nb, int zero_sink,
                     const int32_t* perm, int gate, float gate_q, float gate_temp, void* const* out, void* stream);

/* Replaces forest.soft_gate (forest.py:36-44) on explicit nodes: sm (N, dh) node sums and grp (N, S, dh) their
 * member keys, dtype code `dtype`; out (N, dh) = sm * g * (dh / max(sum g, 1)), g = sigmoid((ml - thr) / gate_temp)
 * with ml the members' mean of log(|x| + 1e-6) per dimension and thr its gate_q quantile over the dimensions. */
int ta_soft_gate(const void* sm, const void* grp, int dtype, int64_t N, int S, int dh, float gate_q,
                 float gate_temp, void* out, void* stream);

/* Replaces the forest descent and key-position step of TreeAttention.sparse_attend (attention.py:73-90, 112-118):
 * per query t of (b, h) (q (Bn, H, T, dh) strided, dtype code `dtype`), the roots of the blocks before t's block
 * scored q . sum (rounded to the dtype), the best min(wmax, width) kept per level with the first bq (per query, or
 * bq_const when bq is NULL) valid, children of the valid kept nodes down to level depth. levels[l]: the level sums
 * of ta_forest_levels; perm: its rank order. Outputs (Bn, H, T, wl) leaf ids / validity and (Bn, H, T, 2 wl) key
 * positions (slot j wl + i: key j of leaf i) with tok = valid and not the sink / t-1 / t-2 of an earlier block.
 * lsel / lselv (arrays of depth + 1 pointers, or NULL): every level's kept ids / validity (Bn, H, T, w_l). */
int ta_forest_select(const void* q, int dtype, int Bn, int H, int T, int dh, int64_t q_sb, int64_t q_sh,
                     int64_t q_st, const void* const* levels, const int32_t* perm, int B, int depth,
                     const int64_t* bq, int bq_const, int wmax, int64_t* leaf, uint8_t* leafv, int64_t* tkey,
                     uint8_t* tok, int32_t* const* lsel, uint8_t* const* lselv, void* stream);

/* Replaces the backward of fastseg.sparse_attn (fastseg.py:80-110 _attn_bwd, 158-170 _SparseAttnFn.backward):
 * from the forward's o and lse (natural log) and the output gradient dout, dq (q's dtype) and the fp32 key / value
 * gradients dk, dv, which are ACCUMULATED (vector atomics, as the reference does; zero them first). All tensors
 * dense: q, o, dout, dq (B, H, T, dh); k, v, dk, dv (B, H, T_kv, dh); cand (B, H, T, Kc), -1 = unused. */
int ta_sparse_attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                       const float* lse, int dtype, int B, int H, int T, int T_kv, int dh, const void* cand,
                       int cand64, int Kc, float scale, void* dq, float* dk, float* dv, void* stream);

/* Replaces fastseg.gather_dot (fastseg.py:118-130, _gather_dot_kernel 34-47): out (B, H, N, C) fp32 =
 * scale * q[b,h,n] . S[b,h,cand[b,h,n,c]] with ids clamped to [0, M-1]. q and S share `dtype`. */
int ta_gather_dot(const void* q, const void* S, int dtype, int B, int H, int N, int M, int C, int dh,
                  int64_t q_sb, int64_t q_sh, int64_t q_st, int64_t s_sb, int64_t s_sh, int64_t s_st,
                  const void* cand, int cand64, float scale, float* out, void* stream);

/* Block form of gather_dot for selections made of whole key blocks (config "gather-dot microbenchmark"):
 * out (B, H, nblk*blk) fp32 = scale * q[b,h] . K[b,h, blocks[b,h,j]*blk + r]; blocks staged into shared
 * memory with bulk copies, nb_cta blocks per CTA (1..64). */
int ta_gather_dot_blocks(const void* q, const void* k, int dtype, int B, int H, int T, int dh, int64_t q_sb,
                         int64_t q_sh, int64_t k_sb, int64_t k_sh, int64_t k_st, const int32_t* blocks, int nblk,
                         int blk, int nb_cta, float scale, float* out, void* stream);

/* Replaces attention_dyn.dedupe (attention_dyn.py:12-17) / fastseg.dedupe_fast (fastseg.py:227-234):
 * keep[r, j] = valid[r, j] and no earlier valid entry of row r has the same value. (rows, Kc) contiguous. */
int ta_dedupe(const int64_t* cand, const uint8_t* valid, uint8_t* keep, int64_t rows, int Kc, void* stream);

/* Replaces SegState.add (engine.py:41-55) for a batch: k, v rows (B, H, dh) of position pos[b] are written
 * into the caches (B, H, cap, dh) and, when pos[b] completes a leaf block, the leaf node and its complete
 * right-spine ancestors are formed. */
int ta_append(const void* k, const void* v, int dtype, int B, int H, int dh, int64_t k_sb, int64_t k_sh,
              int64_t v_sb, int64_t v_sh, void* kc, void* vc, int64_t c_sb, int64_t c_sh, int64_t c_st,
              float* nodes, int64_t n_sb, int64_t n_sh, int cap, int L0, int Lm, const int32_t* pos,
              void* stream);

/* Replaces seg_attend (engine.py:84-120) for a batch, fused: tree descent for the new query, attention over
 * used leaves + sink + window + the new token, append of the new k/v and the incremental tree update.
 * qkv rows (B, 3*H*dh): q at 0, k at k_ofs, v at v_ofs (elements). out rows (B, H*dh). lse / nkeys /
 * sel (B, H, wmax+1) may be NULL. splits: 0 = choose; -1 = persistent pipelined kernel (a selector warp runs
 * the descent of the next (b, h) while the current one streams; for B*H >= #SMs); 1..8 = CTAs per (b, h) of
 * the cluster kernel (split KV merged through distributed shared memory; for small batches).
 * part / part_cnt (may be NULL): scratch of B*H*4*(dh+4) floats and B*H int32 (zero before the first call; the
 * kernel leaves it zero). With it the persistent form (one CTA per SM, e.g. dh 128 bf16 rows) cuts the items of its
 * last, part-empty round into up to 8 parts spread over every CTA (partial states merged by the last part); the
 * outputs are the same up to the fp32 merge order. */
int ta_decode_step(const void* qkv, int dtype, int B, int H, int dh, int64_t qkv_sb, int64_t k_ofs, int64_t v_ofs,
                   void* kc, void* vc, int64_t c_sb, int64_t c_sh, int64_t c_st, float* nodes, int64_t n_sb,
                   int64_t n_sh, int cap, int L0, int Lm, const int32_t* pos, int wmax, int n_tree, int Lw,
                   float scale, void* out, int64_t o_sb, float* lse, int32_t* nkeys, int32_t* sel, int splits,
                   float* part, int32_t* part_cnt, void* stream);

/* The `splits` value ta_decode_step chooses for B*H (b, h) pairs of head dim dh and element type dtype on the
 * current device (-1 = persistent). */
int ta_decode_default_splits(int B, int H, int dh, int dtype);

/* Row kernels of the batched decode step around the attention (callers of the hot path):
 * ta_embed_ln: x[b] = wte[tok[b]] + wpe[pos[b]] (fp32, (B, C)) and h[b] = LayerNorm(x[b]) * w in `dtype`
 *   (reference model.py:75-77 and engine.py:165 embedding, model.py:12-18 LayerNorm without bias).
 * ta_add_ln: x[b] += y[b] (y in `dtype`, NULL = no add), h[b] = LayerNorm(x[b]) * w (engine.py:175-176 residual
 *   adds followed by ln2 / the next layer's ln1).
 * ta_gelu: in-place exact (erf) GELU of n elements (model.py:31 F.gelu), n a multiple of 8.
 * ta_argmax_advance: tok[b] = argmax(logits[b]) (first maximum), pos[b] += 1 (greedy step, phase2.py:61-62). */
int ta_embed_ln(const void* wte, const void* wpe, int dtype, const int64_t* tok, const int32_t* pos, int B, int V,
                int P, int C, const float* w, float eps, float* x, void* h, void* stream);
int ta_add_ln(float* x, const void* y, int dtype, int B, int C, const float* w, float eps, void* h, void* stream);
int ta_gelu(void* x, int dtype, int64_t n, void* stream);
int ta_argmax_advance(const void* logits, int dtype, int B, int V, int64_t* tok, int32_t* pos, void* stream);

/* The decode step's linear layers on the tensor cores (callers of the hot path; reference model.py:21-44 c_attn,
 * c_proj, c_fc + F.gelu, c_mlp; model.py:90 / engine.py:177 the lm_head on the tied embedding; phase2.py:61-62 the
 * greedy argmax). Each replaces one torch matmul of the batched step, plus the elementwise work around it.
 * ta_linear_rows: for rows act (B, K) (row stride act_ld, 16-byte aligned) and an nn.Linear weight w (N, K)
 *   contiguous, both bf16 or both f16, 1 <= B <= 256, K a multiple of 64 x splits:
 *     mode 0 STORE    out (B, N) (row stride out_ld) = act w^T rounded to the dtype, as F.linear;
 *     mode 1 GELU     out = F.gelu of that rounded product (exact erf GELU), rounded;
 *     mode 2 PARTIAL  part (splits, B, N) fp32: the product over each of `splits` K slices, unrounded;
 *     mode 3 ARGMAX   STORE, plus keys (ceil(N / 128), B): per 128-feature tile and row the largest rounded value
 *                     and its first index, packed as (order(value) << 32) | (0xffffffff - index).
 *   Modes 0, 1 and 3 may split K too (more CTAs stream the weight): each split writes its fp32 sums to ws
 *   (ceil(N / 128) x splits x B x 128 floats) and the last split of each 128-feature tile to arrive (counters,
 *   ceil(N / 128) ints, zero before the first call and left zero by every call) adds them in split order and writes
 *   the result, so it does not depend on the order of arrival. N a multiple of 8; outputs 16-byte aligned.
 *   Launched with programmatic dependent launch: the weight stream starts before the previous kernel of the
 *   stream has finished; the rows are read after it has.
 * ta_linear_supported: 1 when ta_linear_rows takes (dtype, B, N, K, splits), else 0 (the caller then uses a
 *   library GEMM).
 * ta_add_splits_ln: x[b] += (sum of part[0 .. splits-1, b] in that order, rounded to `dtype`), then
 *   h[b] = LayerNorm(x[b]) * w (engine.py:175-176: the residual add of a projection's output and the next layer
 *   norm). C a multiple of 8, at most 2048.
 * ta_argmax_finish: tok[b] = the index held by the largest keys[t, b] over the n_tiles tiles, pos[b] += 1. */
int ta_linear_supported(int dtype, int B, int N, int K, int splits);
int ta_linear_rows(const void* act, int64_t act_ld, int dtype, int B, int N, int K, const void* w, int splits, int mode,
                   void* out, int64_t out_ld, float* part, unsigned long long* keys, float* ws, int* counters,
                   void* stream);
int ta_add_splits_ln(float* x, const float* part, int splits, int dtype, int B, int C, const float* w, float eps,
                     void* h, void* stream);
int ta_argmax_finish(const unsigned long long* keys, int n_tiles, int B, int V, int64_t* tok, int32_t* pos,
                     void* stream);

/* The rest of a decode step's transformer block after its attention, and the next block's projection, in ONE
 * launch (reference model.py:21-44 Block.forward after attn: x + c_proj(y), ln_2, c_fc, F.gelu, mlp c_proj,
 * x + mlp; the next block's ln_1 and c_attn; engine.py:161-177 runs this once per decoded token per layer):
 *   x += round(att w_proj^T);            h2 = LayerNorm(x) * ln2_w
 *   fc = round(gelu(round(h2 w_fc^T)));  x += round(fc w_mlp^T)
 *   h = LayerNorm(x) * ln_next_w;        qkv = round(h w_qkv^T)          (when w_qkv is given)
 * att (B, C), h (B, C) and qkv (B, 3C) contiguous in `dtype` (bf16 or f16), x (B, C) fp32 in place; weights as
 * nn.Linear stores them: w_proj (C, C), w_fc (4C, C), w_mlp (C, 4C), w_qkv (3C, C), contiguous 16-bit; ln2_w and
 * ln_next_w (C,) fp32 (LayerNorm without bias, as ta_add_ln). w_qkv and qkv are both NULL after the last block
 * (ln_next_w is then ln_f). 1 <= B <= 128, C a multiple of 128 up to 2048. The layer norms, roundings and GELU are
 * those of ta_add_splits_ln / ta_linear_rows; the fp32 sums of each projection run in a fixed order, so repeated
 * calls give identical results.
 * One CTA per SM; all CTAs are resident together and order the phases through `sync` (sync_words int32, zero
 * before the first call; every call leaves them zero). ws (ws_bytes) holds the projections' fp32 partial sums and
 * the 16-bit rows between phases. Calls that share `sync` or `ws` must not overlap on the GPU. Every wait is
 * bounded: a CTA that gives up records a device error (ta_device_error) and the others end early.
 * Launched with programmatic dependent launch: the weight stream starts before the previous kernel of the stream
 * has finished.
 * ta_block_tail_plan: ws_bytes and sync_words for (dtype, B, C, with_qkv) on the current device, or TA_ERR_ARG
 *   (with the reason) when ta_block_tail does not take the shape. */
int ta_block_tail_plan(int dtype, int B, int C, int with_qkv, int64_t* ws_bytes, int* sync_words);
int ta_block_tail(const void* att, float* x, const void* w_proj, const float* ln2_w, const void* w_fc,
                  const void* w_mlp, const float* ln_next_w, const void* w_qkv, float eps, int dtype, int B, int C,
                  void* h, void* qkv, void* ws, int64_t ws_bytes, int* sync, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TREEATTN_B200_H */
