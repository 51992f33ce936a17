/*
 * saf_api.h -- C ABI of the B200 (sm_100a) sparse-attention hot path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as `void*`, a cudaStream_t), returns a saf_status, allocates no
 * device memory and never synchronises the device (except the functions
 * documented as synchronising).  All work is enqueued on the given stream.
 * An entry point runs on the device that owns its tensors and leaves the
 * calling thread's current CUDA device as it found it.
 *
 * The reference (xiaolong-li1/SparseAttnFunctions, Python + Triton) has no
 * FFI; the Python host package `sparseattnfunctions_b200.special_attentions`
 * binds these symbols with ctypes and keeps the reference's Python names.
 * Each declaration below names the reference function whose work it
 * replaces (path:line inside the reference project).
 *
 * Tensor convention: q, k, v, o are [B, H, S, D] ("HND") with element
 * strides; the D stride must be 1.
 */
#ifndef SAF_API_H
#define SAF_API_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SAF_ABI_VERSION 1

typedef enum saf_status {
  SAF_OK = 0,
  SAF_ERR_SHAPE = 1,       /* inconsistent or unsupported sizes */
  SAF_ERR_DTYPE = 2,       /* unsupported or mismatched element type */
  SAF_ERR_STRIDE = 3,      /* bad stride or pointer alignment */
  SAF_ERR_CUDA = 4,        /* a CUDA runtime call failed */
  SAF_ERR_TIMEOUT = 5,     /* a device-side wait ran out of its budget */
  SAF_ERR_NCCL = 6,        /* reserved for the collective layer */
  SAF_ERR_ARG = 7,         /* null pointer or bad scalar argument */
  SAF_ERR_UNSUPPORTED = 8, /* device is not sm_100 or config has no kernel */
  SAF_ERR_WORKSPACE = 9    /* workspace missing or too small */
} saf_status;

typedef enum saf_dtype { SAF_BF16 = 0, SAF_F16 = 1, SAF_F32 = 2 } saf_dtype;

/* Device status flags (sticky, per device; read with saf_read_device_status). */
#define SAF_DEV_TIMEOUT 0x1u   /* an mbarrier wait gave up */
#define SAF_DEV_BADINDEX 0x2u  /* a CSR column index was out of range and skipped */

/* A [B, H, S, D] tensor view in device memory (strides in elements). */
typedef struct saf_tensor4 {
  void* data;
  int32_t dtype; /* saf_dtype */
  int32_t reserved;
  int64_t B, H, S, D;
  int64_t stride_b, stride_h, stride_s; /* stride_d == 1 */
} saf_tensor4;

/* Block-selection settings for saf_pool_topk. */
typedef struct saf_select_cfg {
  int32_t block_m;            /* query rows per mask block (64 or 128) */
  int32_t block_n;            /* key rows per mask block (64 or 128)   */
  int32_t topk;               /* blocks kept per row by pooled score   */
  int32_t text_blocks_q;      /* row blocks [0, text_blocks_q) are dense */
  int32_t text_blocks_k;      /* columns [0, text_blocks_k) live in every row */
  int32_t force_diag;         /* 1: column i is live in row i            */
  int32_t forced_inside_topk; /* 1: forced columns count toward topk     */
  int32_t reserved;
} saf_select_cfg;

/* ---- library / device ---------------------------------------------- */

/* Self-test of failure detection: launches a one-warp kernel that waits on an
 * mbarrier nothing arrives on; after budget_ns (at most 10 s) the wait gives
 * up and sets SAF_DEV_TIMEOUT, exactly as a stuck wait in any kernel does.
 * Test hook with no reference counterpart. */
int32_t saf_selftest_timeout(uint64_t budget_ns, void* stream);

int32_t saf_abi_version(void);
const char* saf_status_string(int32_t status);
/* SAF_OK when `device` is an sm_100 GPU the kernels were built for. */
int32_t saf_device_check(int32_t device);
/* Budget of every device-side mbarrier wait, in nanoseconds (default 1 s).
 * A wait that runs out sets SAF_DEV_TIMEOUT and the kernel returns early; a
 * wait that is still pending while that flag is set gives up as well. */
void saf_set_wait_budget_ns(uint64_t ns);
uint64_t saf_get_wait_budget_ns(void);
/* Synchronises `device`, returns its sticky status flags, clears them if
 * `clear` is non-zero.  Not for the hot path. */
int32_t saf_read_device_status(int32_t device, uint32_t* flags_out, int32_t clear);

/* ---- (1) block selection --------------------------------------------
 * Mean-pools q and k per block (fp64), scores the pooled blocks
 * (q_mean . k_mean, fp64, ascending d), keeps the top-k columns of every
 * row block (ties: lower column first), forces text rows/columns (and the
 * diagonal when asked) and writes a segmented CSR:
 *   row_ptr [B*H, nbq+1] int32, absolute offsets into col_idx;
 *   head g's entries lie in [g*nbq*nbk, (g+1)*nbq*nbk) (col_idx capacity
 *   B*H*nbq*nbk), columns ascending within a row.
 * mask_out [B*H, nbq, nbk] uint8 and score_out [B*H, nbq, nbk] fp64 are
 * optional (NULL to skip).
 * Replaces: calc_attn_block_sum_efficient (utils/mask_related.py:40-81),
 * get_sparse_attn_mask_from_topk (utils/block_sparse_attn_kernel.py:31-39),
 * the forced text rows/columns of transfer_attn_to_mask
 * (SparseGen_Plus.py:81-82) and get_block_mask's dense padding
 * (utils/mask_related.py:402-403). */
size_t saf_pool_topk_workspace_bytes(const saf_tensor4* q, const saf_tensor4* k,
                                     const saf_select_cfg* cfg);
int32_t saf_pool_topk(const saf_tensor4* q, const saf_tensor4* k, const saf_select_cfg* cfg,
                      int32_t* row_ptr, int32_t* col_idx, uint8_t* mask_out, double* score_out,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Block selection without a workspace argument.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory when
 * they call in (memory planned once and frozen, plugin slots that receive
 * only their inputs and outputs, loops that must not synchronise on
 * cudaMalloc).  Same results as saf_pool_topk; the scratch comes from a
 * static SAF_STATIC_SCRATCH_BYTES device array that every GPU loading this
 * library holds until the process exits.  Returns SAF_ERR_WORKSPACE when the
 * problem needs more scratch than that (saf_pool_topk_workspace_bytes tells
 * how much).  Allocates nothing.  The first call on each device looks up the
 * array's device address (make that first call before any stream capture).
 * All calls share the array: calls that overlap on the GPU race. */
#define SAF_STATIC_SCRATCH_BYTES (16u << 20) /* 16 MiB */
int32_t saf_pool_topk_noalloc(const saf_tensor4* q, const saf_tensor4* k,
                              const saf_select_cfg* cfg, int32_t* row_ptr, int32_t* col_idx,
                              uint8_t* mask_out, double* score_out, void* stream);

/* Dense boolean block mask [BH, nbq, nbk] (uint8, element strides
 * stride_bh / stride_row, column stride 1) -> segmented CSR as above.
 * Replaces the dense-mask walk of _fwd_kernel
 * (utils/block_sparse_attn_kernel.py:167-199), which reads every mask bit. */
int32_t saf_mask_to_csr(const uint8_t* mask, int64_t BH, int32_t nbq, int32_t nbk,
                        int64_t stride_bh, int64_t stride_row, int32_t* row_ptr,
                        int32_t* col_idx, void* stream);

/* Energy-threshold block selection (SparseGen_Plus's adaptive density).
 * in: fp64 [BH, nbq, nbk] contiguous -- the estimated attention mass per key
 * block when is_mass != 0, else mean-pooled scores (saf_pool_topk's scores)
 * turned into mass_j = n_j * exp(scale * s_j - max scale * s) with n_j the
 * tokens of key block j (block_n, last block Sk - (nbk-1)*block_n).  Per
 * row: sort descending (ties to the lower column), keep the prefix that
 * ends before the first position where the fp64 running sum reaches
 * threshold * total (all if none), clamped to [min_retain, max_retain];
 * rows / columns < text_blocks forced.  Writes the uint8 block mask
 * [BH, nbq, nbk] (saf_mask_to_csr makes the CSR) and, if mass_out is not
 * null, the mass used.  nbk <= 1024.
 * Replaces: transfer_attn_to_mask(mode="energy") (SparseGen_Plus.py:12-84). */
int32_t saf_energy_select(const double* in, int32_t is_mass, int64_t BH, int32_t nbq, int32_t nbk,
                          int32_t block_n, int64_t Sk, double scale, double threshold,
                          int32_t min_retain, int32_t max_retain, int32_t text_blocks,
                          double* mass_out, uint8_t* mask, void* stream);

/* Adaptive top-k block selection on the same input: per row, with the mass
 * sorted descending (ties to the lower column) and E = the fp64 running sum
 * of the first init_k blocks, k = init_k; if E < 0.6 x total, k = min(3k,
 * nbk); then if E < 0.9 x total, k = min(k / 3 * 2, nbk) (integer division,
 * on the updated k); the first k sorted blocks are kept and rows / columns
 * < text_blocks forced.  1 <= init_k <= nbk (the caller turns a fraction
 * into a count as the reference does: int(nbk * init_k)).
 * Replaces: transfer_attn_to_mask(mode="topk") (SparseGen_Plus.py:28-50). */
int32_t saf_topk_adaptive_select(const double* in, int32_t is_mass, int64_t BH, int32_t nbq,
                                 int32_t nbk, int32_t block_n, int64_t Sk, double scale, int32_t init_k,
                                 int32_t text_blocks, double* mass_out, uint8_t* mask, void* stream);

/* ---- (2) block-sparse attention -------------------------------------
 * o[b,h,i,:] = sum_{j live} softmax_j(sm_scale * q_i . k_j + bias_j) v_j
 * over the key blocks listed in the CSR row of query block i / block_m.
 * bf16 / f16: tcgen05 + TMEM + TMA kernel (D = 64), fp32 accumulation,
 * output in the input type.  f32: CUDA-core kernel in full fp32.
 * kv_bias (nullable): fp32 additive bias per key column, read at
 * kv_bias[g * kv_bias_stride_bh + j] for head g = b*H + h (stride 0
 * broadcasts one row).  Rows with no live block give NaN (0/0), as the
 * reference kernel does.
 * col_capacity bounds every col_idx read (entries past it are ignored).
 * lead_rows: query blocks [0, lead_rows) of every head are scheduled before
 * all others -- pass the number of dense (text) rows, whose block lists are
 * the longest, so they do not start last and stretch the tail; 0 keeps
 * head-major order.  With few heads per GPU a lead tile would outlast the
 * rest of the launch, so their key blocks are split over up to 8 work items
 * whose partial rows are merged by the last of them (fp32 partials in a
 * static 16 MiB per-device buffer: launches with lead_rows > 0 on one
 * device must not overlap; launches whose partials would not fit run
 * unsplit).  Results do not depend on it beyond fp32 rounding.
 * Each launch takes one of 64 per-device tile-counter slots, round-robin
 * at launch time, and leaves it at zero when it ends: launches ordered on
 * one stream, or fewer than 64 in flight at once, never share a live slot.
 * A launch captured in a CUDA graph keeps its slot for every replay, so a
 * replay must not overlap other attention launches of this library on the
 * same device.
 * Replaces: _forward / _fwd_kernel / _fwd_kernel_inner /
 * block_sparse_triton_fn (utils/block_sparse_attn_kernel.py:52-293) and the
 * bias path of MergeAttention.forward (MergeAttention.py:33-49). */
int32_t saf_bsa_fwd(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                    const saf_tensor4* o, const int32_t* row_ptr, const int32_t* col_idx,
                    int64_t col_capacity, int32_t block_m, int32_t block_n,
                    const float* kv_bias, int64_t kv_bias_stride_bh, float sm_scale,
                    int32_t lead_rows, void* stream);

/* saf_bsa_fwd with per-query-row key intervals: row_ranges (nullable,
 * 16-byte aligned int32 [Sq, 4], shared by every head) limits the keys of
 * query row r to [x, y) U [z, w); keys outside are masked like keys past
 * Sk.  The CSR must list every block that some row of the query block can
 * see (a superset is fine).  Not combinable with kv_bias.
 * Replaces: the frame-band masks of SmartAttention.attention_with_mask and
 * its flex_attention block mask (SmartAttention.py:30-43,130-151). */
int32_t saf_bsa_fwd_ranges(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                           const saf_tensor4* o, const int32_t* row_ptr, const int32_t* col_idx,
                           int64_t col_capacity, int32_t block_m, int32_t block_n,
                           const float* kv_bias, int64_t kv_bias_stride_bh, float sm_scale,
                           int32_t lead_rows, const int32_t* row_ranges, void* stream);

/* ---- frame-scope masks (frame x frame sparsity on the unpadded sequence)
 * The sequence is [text_len text tokens | frames x frame_len video tokens].
 *
 * saf_frame_mask: the frame x frame attention map of a sampled subset --
 * every text token and, in every frame, the same n spatial positions
 * spatial[0..n) (int32 in [0, frame_len)) -- and its per-head 90 %-style
 * energy mask.  logits = sm_scale * q_s . k_s (+ log(n / frame_len), as a
 * float32, on the text keys), softmax over the sampled keys, map[f1, f2] =
 * the video-video probability of frame pair (f1, f2) summed over the frame's
 * sampled queries / n; per head the flattened map sorted in descending
 * order keeps every entry ranked at or before the first position whose
 * cumulative sum reaches threshold x the total.  Outputs: bits_out [B*H,
 * frames] uint32 (bit f2 of word f1 = frame f2 visible to frame f1),
 * optional mask_out [B*H, frames, frames] uint8 and map_out fp64.
 * frames <= 32, n <= frame_len, D = 64 or 128; workspace of
 * saf_frame_mask_workspace_bytes.  An out-of-range spatial entry sets
 * SAF_DEV_BADINDEX and reads position 0.
 * Replaces: generate_attention_mask_frame_scope
 * (utils/mask_related.py:194-245), which draws the spatial sample itself. */
size_t saf_frame_mask_workspace_bytes(int64_t BH, int32_t frames, int32_t n, int32_t text_len,
                                      int32_t D);
int32_t saf_frame_mask(const saf_tensor4* q, const saf_tensor4* k, const int32_t* spatial, int32_t n,
                       int32_t text_len, int32_t frames, int32_t frame_len, float sm_scale,
                       double threshold, void* workspace, size_t workspace_bytes, double* map_out,
                       uint8_t* mask_out, uint32_t* bits_out, void* stream);

/* Frame masks -> segmented CSR over block_m x block_n blocks of the
 * unpadded sequence (S = text_len + frames x frame_len, frames < 32,
 * frame_len >= block_n): a query block holding a text row lists every key
 * block; any other lists the key blocks holding a text key or a key of a
 * frame that one of its frames sees.
 * Replaces: get_block_mask (utils/mask_related.py:397-404), whose kron of
 * the frame mask with a per-frame block mask needs frame-aligned padding. */
int32_t saf_frame_csr(const uint32_t* bits, int64_t BH, int32_t text_len, int32_t frames,
                      int32_t frame_len, int64_t S, int32_t block_m, int32_t block_n, int32_t* row_ptr,
                      int32_t* col_idx, void* stream);

/* saf_bsa_fwd under frame masks: inside every visited block, a video query
 * of frame f1 of head g sees only the text keys and the keys of the frames
 * set in frame_bits[g * frames + f1]; text queries see every key.  16-bit
 * inputs, Sq = Sk = text_len + frames x frame_len, frame_len >= block_n.
 * Replaces: block_sparse_triton_fn on the padded and randomly truncated
 * layout of BlockSparseAttention.forward_backup (block_mask_attn.py:11-20,
 * utils/mask_related.py:87-187). */
int32_t saf_bsa_fwd_frames(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                           const saf_tensor4* o, const int32_t* row_ptr, const int32_t* col_idx,
                           int64_t col_capacity, int32_t block_m, int32_t block_n,
                           const uint32_t* frame_bits, int32_t text_len, int32_t frames,
                           int32_t frame_len, float sm_scale, int32_t lead_rows, void* stream);

/* Attention with a pooled attention map.  Runs the block-sparse attention
 * (16-bit inputs, no key bias) and writes pool_out [B*H, nbp, nbk] fp32,
 * nbp = ceil(Sq / pool_block), nbk = ceil(Sk / block_n):
 *   pool_out[g, i, j] = max over query rows r of block i of
 *                       exp2(R[r, j] - lse_r),
 * R[r, j] = row r's largest logit in key block j (log2 units, sm_scale
 * folded in; -inf for blocks the row does not visit), lse_r = the row's
 * log2-sum-exp; then every row of pool_out is divided by its sum.
 * pool_block is 128, or 64 with 64-row mask blocks (block_m 64): a pooled
 * row is one 128-row query tile of the kernel or one half of it, reduced in
 * the tile's epilogue (no pass over an R array in HBM).
 * workspace: caller-allocated, at least saf_bsa_pool_workspace_bytes(B*H,
 * Sq, nbk) bytes (each persistent CTA's R of its current tile, fp32; sized
 * for the current device).  fp32 inputs: SAF_ERR_UNSUPPORTED.
 * Replaces: attn_with_pooling / _attention_pooling.forward and _attn_fwd
 * (special_attentions/utils/attn_pooling_kernel.py:25-97,106-264; the
 * non-causal case, whose query and key blocks are both block_size). */
int64_t saf_bsa_pool_workspace_bytes(int64_t BH, int64_t Sq, int32_t nbk);
int32_t saf_bsa_fwd_pool(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                         const saf_tensor4* o, const int32_t* row_ptr, const int32_t* col_idx,
                         int64_t col_capacity, int32_t block_m, int32_t block_n, float sm_scale,
                         int32_t lead_rows, int32_t pool_block, void* workspace,
                         int64_t workspace_bytes, float* pool_out, void* stream);

/* ---- (3) ToMe token merging -----------------------------------------
 * Output buffers of a bipartite matching.  Positions refer to the src list
 * a_idx (length Ns) and the dst list b_idx (length Nd) of video tokens.
 *   unm_idx   [B, Ns-r]  src positions kept, in edge order (node_max desc)
 *   src_idx   [B, r]     src positions merged, in edge order
 *   dst_idx   [B, r]     dst position each of them merges into
 *   counter   [B, Nd]    1 + number of src merged into each dst
 *   dst_ptr   [B, Nd+1]  CSR over dst_src (offsets within the batch row)
 *   dst_src   [B, r]     merged src positions grouped by dst, edge order
 *   token_map [B, N]     (nullable) merged-sequence row of every video token
 *   log_count [B, Nd]    (nullable) log(counter) in fp32, the proportional-
 *                        attention bias of the dst columns
 *   node_max  [B, Ns]    (nullable) exact fp64 best cosine of every src
 *   node_idx  [B, Ns]    (nullable) its dst position */
typedef struct saf_tome_plan {
  int32_t* unm_idx;
  int32_t* src_idx;
  int32_t* dst_idx;
  int32_t* counter;
  int32_t* dst_ptr;
  int32_t* dst_src;
  int32_t* token_map;
  float* log_count;
  double* node_max;
  int32_t* node_idx;
} saf_tome_plan;

/* Bipartite soft matching of the video tokens of metric [B, N, C]
 * (bf16/f16, element strides stride_b / stride_n, C contiguous): cosine
 * similarity of every src (a_idx) with every dst (b_idx) token, best dst per
 * src, src sorted by it, the first r merged.  Exact contract: fp64 cosine of
 * the input values, arg-max ties to the lower dst position, sort ties to the
 * lower src position.  Tensor cores score all pairs, no score matrix is
 * written to memory.  r larger than Ns is clamped to Ns.
 * Replaces: bipartite_soft_matching_video (utils/merge_unmerge.py:34-116). */
size_t saf_tome_match_workspace_bytes(int64_t B, int64_t Ns, int64_t Nd, int64_t C, int32_t r);
int32_t saf_tome_match(const void* metric, int32_t dtype, int64_t B, int64_t N, int64_t C,
                       int64_t stride_b, int64_t stride_n, const int32_t* a_idx, int64_t Ns,
                       const int32_t* b_idx, int64_t Nd, int32_t r, const saf_tome_plan* plan,
                       void* workspace, size_t workspace_bytes, void* stream);

/* The matching metric of MergeAttention: for every (b, h) and video token
 * n (rows text_len.. of k / v [B, H, S, D], bf16 / f16), out[b*H + h, n] =
 * [k, |k|, v, |v|] (2D + 2 values, contiguous [B*H, S - text_len, 2D + 2]);
 * D even, at most 128.  Each norm is the fp64 sqrt of an fp64 sum of
 * squares in a fixed order (lane l of a warp sums the pairs
 * x[2w]^2 + x[2w+1]^2 of words w = l, l + 32 in ascending order, the lanes
 * combine by the xor butterfly 16, 8, 4, 2, 1), rounded once to the 16-bit
 * type.
 * Replaces: the metric of MergeAttention.forward (MergeAttention.py:26-31). */
int32_t saf_tome_kv_metric(const saf_tensor4* k, const saf_tensor4* v, int32_t text_len, void* out,
                           void* stream);

/* merge: x [B, text_len + N, C] -> out [B, text_len + (Ns-r) + Nd, C]:
 * text rows copied, then the kept src tokens (unm_idx order), then every dst
 * token averaged with the src merged into it (fp32 sum in edge order /
 * counter; the reference's scatter_reduce "mean" with include_self).
 * Replaces: merge (utils/merge_unmerge.py:119-135). */
int32_t saf_tome_merge(const void* x, void* out, int32_t dtype, int64_t B, int64_t C,
                       int64_t x_stride_b, int64_t x_stride_n, int64_t o_stride_b,
                       int64_t o_stride_n, int32_t text_len, const int32_t* a_idx, int64_t Ns,
                       const int32_t* b_idx, int64_t Nd, int32_t r, const saf_tome_plan* plan,
                       void* stream);

/* unmerge: y [B, text_len + (Ns-r) + Nd, C] -> out [B, text_len + N, C]:
 * every video token reads its merged row (token_map).
 * Replaces: unmerge (utils/merge_unmerge.py:137-154). */
int32_t saf_tome_unmerge(const void* y, void* out, int32_t dtype, int64_t B, int64_t C,
                         int64_t y_stride_b, int64_t y_stride_n, int64_t o_stride_b,
                         int64_t o_stride_n, int32_t text_len, int64_t N, const int32_t* token_map,
                         void* stream);

/* Token permutation / padding of [B, H, S, D] tensors (element strides, D
 * contiguous) into [B, H, S_out, D]: out[g, s, :] = x[g, perm[s], :] for
 * s < S_out, a zero row where perm[s] == -1, for the flat heads g = b*H + h
 * listed in heads[0..n_heads) (every head when heads is null).  Other perm
 * entries outside [0, S) or heads outside [0, B*H) set SAF_DEV_BADINDEX in
 * the device status word and are skipped.
 * Replaces: process / process_back of SmartAttention (SmartAttention.py:
 * 16-41), the (t, h, w) <-> (h, w, t) reordering of the video tokens, and
 * preprocess / process_out_back of SildingTileAttention
 * (SildingTileAttention.py:106-136) with every tile padded to a block. */
int32_t saf_permute_tokens(const void* x, void* out, int32_t dtype, int64_t B, int64_t H, int64_t S,
                           int64_t S_out, int64_t D, int64_t x_sb, int64_t x_sh, int64_t x_ss,
                           int64_t o_sb, int64_t o_sh, int64_t o_ss, const int32_t* perm,
                           const int32_t* heads, int64_t n_heads, void* stream);

/* Ulysses sequence <-> head layout for the all-to-all of sequence-sharded
 * attention.  Sequence-sharded tensors are [B, s, H, D] (element strides
 * stride_b / stride_s / stride_h, D contiguous, D * element size a multiple
 * of 16 bytes, 16-byte aligned rows); head_off (host array, P + 1 entries,
 * head_off[0] = 0, head_off[P] = H) gives each peer's contiguous head range.
 * pack writes T (<= 4) tensors into buf as P chunks back to back, chunk j =
 * heads of peer j as [s, B, T, h_j, D]; unpack is the inverse.  After an
 * all-to-all of these chunks a peer holds [S, B, T, h, D]: each tensor a
 * strided [B, h, S, D] view for saf_bsa_fwd / saf_pool_topk.
 * Replaces: no reference function (the reference runs on one GPU); these
 * are the layout steps around the NCCL all-to-all of sequence-sharded runs. */
int32_t saf_ulysses_pack(void* const* seq, int32_t T, int32_t dtype, int64_t B, int64_t s, int64_t H,
                         int64_t D, int64_t stride_b, int64_t stride_s, int64_t stride_h,
                         const int32_t* head_off, int32_t P, void* buf, void* stream);
int32_t saf_ulysses_unpack(const void* buf, int32_t T, int32_t dtype, int64_t B, int64_t s, int64_t H,
                           int64_t D, int64_t stride_b, int64_t stride_s, int64_t stride_h,
                           const int32_t* head_off, int32_t P, void* const* seq, void* stream);

/* ---- (6) local + global keys (LocalGlobalAttention) -------------------
 * Row gather: out[ob, h, s, :] = x[src / Sx, h, src % Sx, :] with
 * src = idx[ob * So + s] (int64, flattened (batch, row) of x); src < 0
 * writes a zero row, src >= Bx * Sx a zero row and SAF_DEV_BADINDEX.  D x
 * element size a multiple of 16 bytes, pointers 16-byte aligned, strides in
 * elements (multiples of 16 bytes).  Duplicated sources are allowed.
 * Replaces: transform_q / transform_kv_v1 / transform_output
 * (special_attentions/LocalGlobalAttention.py:212-245): the rearranges and
 * the torch.gather of k / v by each (patch, batch) key list. */
int32_t saf_gather_rows(const void* x, int32_t dtype, int64_t Bx, int64_t H, int64_t Sx, int64_t D,
                        int64_t x_sb, int64_t x_sh, int64_t x_ss, void* out, int64_t Bo, int64_t So,
                        int64_t o_sb, int64_t o_sh, int64_t o_ss, const int64_t* idx, void* stream);

/* Probe mass of sampled query rows: qs [B, H, R, 64] holds the R sampled
 * rows of every head (gathered), k [B, H, Sk, 64], both bf16 or both f16.
 * mass_out [B, Sk] fp64 = round16(sum over heads and rows of
 * round16(softmax_keys(round16(qs . k) / 8))), round16 = rounding to the
 * input type, sums in fp32 in a fixed order (the reference's 16-bit matmul,
 * softmax and sum).  tcgen05 kernel; workspace of
 * saf_probe_workspace_bytes(B, H, Sk, R) bytes.
 * Replaces: probe_solver._probe_num up to the masked_fill
 * (special_attentions/LocalGlobalAttention.py:50-57). */
size_t saf_probe_workspace_bytes(int64_t B, int64_t H, int64_t Sk, int32_t n_samp);
int32_t saf_probe_mass(const saf_tensor4* qs, const saf_tensor4* k, void* workspace,
                       size_t workspace_bytes, double* mass_out, void* stream);

/* Attention over per-batch key lists: o[b, h, i] = softmax over the keys
 * j < key_len of (sm_scale * q[b, h, i] . k[sb, h, key_list[b, j]]) applied
 * to v[sb, h, key_list[b, j]], sb = key_batch[b] -- every listed key once
 * per listing (a repeated key counts twice, as the reference's gather +
 * SDPA).  q / o [Bq, H, Sq, 64], k / v [B_src, H, S_src, 64] bf16 or f16 with
 * contiguous rows (they are read as one array of 64-element rows by TMA
 * gather4 loads, four key rows per load, no gathered copy in HBM);
 * key_list [Bq, key_len] int32, key_batch [Bq] int32 (out-of-range entries
 * read row 0 and set SAF_DEV_BADINDEX).  Tensor-core kernel (sm_100a).
 * Replaces: transform_kv_v1 + attention_video of LocalGlobalAttention
 * (special_attentions/LocalGlobalAttention.py:219-238, 207-210): the
 * torch.gather of k / v by each (patch, batch) key list and the SDPA over
 * the gathered rows. */
int32_t saf_bsa_fwd_keys(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                         const saf_tensor4* o, const int32_t* key_list, int32_t key_len,
                         const int32_t* key_batch, float sm_scale, void* stream);

/* Masked top-n: for row r = p * B + b of out [P * B, n] int32, the n keys of
 * largest mass[b, :] among those with local_mask[p, key] == 0 (uint8
 * [P, Sk]), ties to the lower key, in ascending key order.  n <= the
 * unmasked keys of every row.
 * Replaces: the masked_fill, descending sort and slice of
 * probe_solver._probe_num (special_attentions/LocalGlobalAttention.py:58-62). */
int32_t saf_masked_topn(const double* mass, const uint8_t* local_mask, int64_t B, int64_t P, int64_t Sk,
                        int32_t n, int32_t* out, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SAF_API_H */
