/*
 * specverify.h -- C ABI of the B200 (sm_100a) tree-verification library.
 *
 * One shared library (libspecverify.so) holds every kernel of DiffSpec's
 * target-side tree-verification hot path.  All entry points:
 *   - are extern "C", take plain device pointers, element strides and sizes,
 *     and a cudaStream_t (passed as void*; NULL = legacy default stream);
 *   - never allocate or free device memory: the caller passes outputs and any
 *     workspace (sized by the *_workspace_size queries);
 *   - are stream-ordered and never synchronise the host;
 *   - return TV_OK (0) or a negative tv_status; they never trap on the GPU.
 *     Argument errors are detected on the host before any launch; errors the
 *     kernels detect (bad parent pointers, page ids out of range) are written
 *     to a status word in device memory that the caller reads back.
 *
 * Element strides are in elements of the tensor's own dtype; the innermost
 * (head_dim) stride must be 1.  Byte strides are named *_bytes.
 *
 * Reference interfaces replaced (paths inside the reference package
 * ``diffspec``):
 *   tv_verify_attn        diffspec/runtime/tree_attention.py:414-446
 *                         (prefix_attention_forward), :462-539
 *                         (tree_attention_forward), and the merge at
 *                         diffspec/runtime/llama_target_model.py:835-864;
 *                         diffspec/runtime/bundle_verifier.py:166-257
 *                         (FusedBundleVerifier.verify_bundle) and :341-366
 *                         (PagedBundleVerifier.verify_bundle_paged)
 *   tv_merge_partials     diffspec/runtime/tree_attention.py:535-539 (LSE merge)
 *   tv_pack_mask          diffspec/runtime/tree_attention.py:449-460
 *   tv_accept             diffspec/draft/tree_verification.py:100-182
 *   tv_compact_contig     diffspec/draft/tree_verification.py:197-217,
 *                         diffspec/runtime/cache_state.py:38-50
 *   tv_copy_pages,
 *   tv_compact_paged      diffspec/core/kv_cache/paged_kv.py:168-223 (COW)
 *   tv_arena_gather       diffspec/core/kv_cache/chunk_arena.py:126-173
 *   tv_gather_page_table  diffspec/core/kv_cache/chunk_arena.py:86-178 (zero-copy form)
 *   tv_rope_append        diffspec/runtime/llama_target_model.py:429-474 (RoPE)
 *                         and diffspec/runtime/cache_state.py:52-66 (KVCache.cat)
 *   tv_lmhead_accept      diffspec/draft/diffspec_model.py:229-231 (lm_head) and
 *                         diffspec/draft/tree_verification.py:100-162
 *   tv_tree_finalize      diffspec/runtime/draft_tree.py:188-260 and
 *                         diffspec/draft/diffspec_model.py:620-624 (root prepend)
 *   tv_chunk_select,
 *   tv_gather_rows        diffspec/draft/draft_network.py:1514-1612 (retrieval)
 */
#ifndef SPECVERIFY_H_
#define SPECVERIFY_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------- */
enum tv_status {
  TV_OK = 0,
  TV_ERR_SHAPE = -1,       /* inconsistent or unsupported sizes           */
  TV_ERR_DTYPE = -2,       /* unsupported element type                    */
  TV_ERR_ALIGN = -3,       /* pointer / stride not 16-byte aligned        */
  TV_ERR_LAUNCH = -4,      /* CUDA launch or runtime error                */
  TV_ERR_WORKSPACE = -5,   /* workspace missing or too small              */
  TV_ERR_INPUT = -6,       /* invalid input values (device-detected)      */
  TV_ERR_UNSUPPORTED = -7, /* valid request this build does not handle    */
  TV_ERR_NULL = -8         /* required pointer is NULL                    */
};

enum tv_dtype { TV_BF16 = 0, TV_F16 = 1, TV_F32 = 2 };

/* Human-readable text for a status code (static storage). */
const char* tv_status_string(int status);
/* Library version, e.g. "specverify 0.1 sm_100a". */
const char* tv_version(void);
/* Text of the last CUDA error an entry point saw on this host thread. */
const char* tv_last_cuda_error(void);

/* ---- verify attention ------------------------------------------------
 *
 * For every batch b, query row m (tree node) and query head h (KV head
 * h / (heads / kv_heads)):
 *
 *   out[b,m,h,:] = softmax_n(scale * q[b,m,h,:] . k[b,n,hk,:]) @ v[b,n,hk,:]
 *   lse[b,m,h]   = log sum_n exp(scale * q . k)        (natural log)
 *
 * over the keys n < len_b visible to row m: every key before
 * tail_b = len_b - mask_len, and key tail_b + j when bit j of the row's mask
 * is set (word j / 64, bit j % 64 of mask[b * mask_sb + m * mask_sm + ...]).
 * len_b = kv_lens[b] if kv_lens != NULL, else num_keys.
 * A row with no visible key gets out = 0 and lse = -inf.
 *
 * KV addressing:
 *   contiguous (page_table == NULL): key n of (b, hk) starts at
 *       k + b * k_sb + n * k_sn + hk * k_sh;
 *   paged: page = page_table[b * pt_sb + n / page_size]; the key starts at
 *       k + page * k_sb + hk * k_sh + (n % page_size) * k_sn
 *     (k_sb is the page stride); a negative page id reads as zeros.
 * v uses its own v_* strides the same way.
 *
 * Optional epilogues: lse (fp32, strided) and, when aux_lse != NULL,
 *   weight[b,m,h] = (dtype) sigmoid(aux_lse[b,m,h] - lse[b,m,h])
 * (the merge weight of tree_attention.py:539).
 * out_f32 != 0 writes out in fp32 instead of `dtype`.
 *
 * Work is split over the keys (split-KV); the partial (O, lse) pairs live in
 * the caller's workspace and are merged by log-sum-exp in a second kernel.
 */
typedef struct tv_attn_args {
  int32_t dtype;                 /* TV_BF16 or TV_F16 for q, k, v, out      */
  int32_t batch, rows, heads, kv_heads, head_dim;
  float scale;                   /* softmax scale, usually 1/sqrt(head_dim) */
  const void* q;
  int64_t q_sb, q_sm, q_sh;
  const void* k;
  const void* v;
  int64_t k_sb, k_sn, k_sh;
  int64_t v_sb, v_sn, v_sh;
  const int32_t* page_table;     /* NULL = contiguous KV                    */
  int64_t pt_sb;
  int32_t page_size;
  int32_t num_pages;             /* physical pages in the pool (bounds check)*/
  const int32_t* kv_lens;        /* optional per-batch key counts (device)  */
  int32_t num_keys;
  int32_t mask_len;              /* keys gated by the bitmask (0 = none)    */
  const uint64_t* mask;
  int64_t mask_sb, mask_sm;
  void* out;
  int64_t o_sb, o_sm, o_sh;
  int32_t out_f32;
  float* lse;                    /* optional                                */
  int64_t lse_sb, lse_sm, lse_sh;
  const float* aux_lse;          /* optional: prefix LSE for the weight     */
  int64_t aux_sb, aux_sm, aux_sh;
  void* weight;                  /* required when aux_lse != NULL           */
  int64_t w_sb, w_sm, w_sh;
  int32_t num_splits;            /* 0 = choose automatically                */
  int32_t kernel;                /* bits 0-3: 0 auto, 1 warp-MMA, 2 tcgen05
                                    only (TV_ERR_UNSUPPORTED when the request
                                    does not fit it);
                                    bit 4 (16): softmax weights as a hi+lo
                                    16-bit pair in the PV product (automatic
                                    for num_keys <= 4096);
                                    tv_verify_attn_sharded only: bit 5 (32)
                                    owner exchange, bit 6 (64) push to every
                                    peer (default: push below 4 ranks,
                                    owner from 4 on);
                                    bit 7 (128): tcgen05 path on a paged
                                    pool loads each 64-dim half of a page
                                    row as its own TMA box (default: one box
                                    for both halves when the pool's page and
                                    head strides allow it)                 */
  void* workspace;
  size_t workspace_bytes;
  int32_t* status;               /* optional device word, zeroed by the caller;
                                    set nonzero if a kernel had to abandon a
                                    wait (its output rows are then NaN)     */
  const uint8_t* mask_words_full;/* optional, [batch][mask words] from
                                    tv_mask_word_summary: 1 where every row's
                                    mask word is all ones, so the tcgen05
                                    kernel skips masking key tiles made only
                                    of such words (same result, less work) */
  int64_t mask_words_full_sb;
} tv_attn_args;

int tv_attn_workspace_size(const tv_attn_args* args, size_t* bytes);
int tv_verify_attn(const tv_attn_args* args, void* stream);

/* The plan tv_verify_attn would run for `args` (host only, nothing launched):
 * info[0] = kernel (1 warp-MMA, 2 tcgen05), info[1] = key splits,
 * info[2] = 1 when the tcgen05 kernel loads whole-head (both 64-dim halves)
 * TMA boxes, info[3] = 1 when the warp-MMA kernel runs split-P.  No
 * counterpart in the reference (its kernel choice is fixed per call site,
 * llama_target_model.py:836-845). */
int tv_attn_describe(const tv_attn_args* args, int32_t* info);

/* tv_verify_attn without a caller workspace: no counterpart in the reference
 * (its attention allocates its temporaries per call).  The split partials
 * live in a fixed 24 MiB device array inside this library, so the call
 * allocates nothing; args->workspace is ignored.  Limits: a request whose
 * partials need more than 24 MiB (see tv_attn_workspace_size) returns
 * TV_ERR_WORKSPACE; calls on the same device share the array and must not
 * overlap; the first call on each device resolves the array's address and
 * must come before any stream capture. */
int tv_verify_attn_static(const tv_attn_args* args, void* stream);

/* Merge `parts` partial attentions over disjoint key sets (split-KV or one
 * per rank of a sequence-sharded cache):
 *   parts_o   [parts][rows][head_dim] fp32, each normalised over its keys
 *   parts_lse [parts][rows] fp32 natural-log LSE
 * writes out [rows][head_dim] (out_dtype) and, if out_lse != NULL, the merged
 * LSE [rows].  Part p of row r is parts_o + p * part_stride + r * head_dim. */
int tv_merge_partials(int32_t parts, int64_t rows, int32_t head_dim,
                      const float* parts_o, int64_t part_stride_o,
                      const float* parts_lse, int64_t part_stride_lse,
                      int32_t out_dtype, void* out, float* out_lse, void* stream);

/* ---- sequence-sharded verify over NVLink peer memory ---------------------
 * No counterpart in the reference (it attends the whole prefix on one device,
 * llama_target_model.py:839-845, and has no multi-GPU code).  One process per
 * GPU; each rank holds a contiguous shard of the keys (the rank holding the
 * tree also its M tree keys and the bitmask).
 *
 * Exchange buffer: tv_sharded_exchange_bytes(world, rows, head_dim) bytes per
 * rank, rows = batch * heads * rows_per_sequence (query rows), allocated so
 * that every rank can address every other rank's buffer (symmetric / IPC
 * memory), 16-byte aligned and zeroed before the first step.  It holds two
 * slots of `world` partials (O and LSE, one 8-byte word per value), the
 * final rows of owner mode and this rank's step counts.  Use one buffer per
 * (world, rows, head_dim): the layout depends on all three.
 *
 * tv_verify_attn_sharded: `args` is this rank's request exactly as for
 * tv_verify_attn (args->num_keys = this shard's keys) except that out / lse /
 * aux_lse / weight receive the MERGED result over all ranks' shards, and
 * args->workspace holds this rank's split partials
 * (tv_verify_attn_sharded_workspace_size bytes).  It launches the attention
 * kernel, then one kernel that combines this rank's split partials and
 * exchanges them over NVLink as 8-byte words that carry the value (fp32 bits,
 * low half) and the step number (high half): an aligned 64-bit store is
 * single-copy atomic, so the reader polls the data itself -- no flags, no
 * fences.  Waits are bounded: 2 s, then *args->status = 8 and NaN rows.
 * Push mode: the partial goes into every peer's buffer and every rank
 * merges all partials.  Owner mode: each row block's partials go to the rank
 * that owns it, which merges them and stores the final rows into every other
 * rank's buffer (about 4 (W-1)/W partials of NVLink bytes per rank instead of
 * 2 (W-1), for a second hop).  Merges run by log-sum-exp in rank order:
 * every rank gets bit-identical outputs.  args->kernel bits 5 / 6 pick the
 * mode (default: push below 4 ranks, owner from 4 on).
 * A word is accepted only when it carries this call's step: a later step
 * means a peer gave up on this rank and moved on, and the rows are flagged
 * (status 8, NaN) rather than merged.
 * bases[r] = rank r's exchange buffer as mapped in this process (world <= 8);
 * exchange_bytes = the size of each (exactly tv_sharded_exchange_bytes for
 * this request's world, rows and head_dim, else TV_ERR_WORKSPACE before any
 * launch).  Every rank must make the same sequence of calls with the same
 * shapes; successive calls alternate the buffer's two slots by themselves. */
int tv_sharded_exchange_bytes(int32_t world, int64_t rows, int32_t head_dim, int64_t* bytes);
int tv_verify_attn_sharded_workspace_size(const tv_attn_args* args, size_t* bytes);
int tv_verify_attn_sharded(const tv_attn_args* args, int32_t world, int32_t rank, const void* const* bases,
                           int64_t exchange_bytes, void* stream);

/* ---- masks --------------------------------------------------------------
 * Pack a [batch][rows][cols] keep-mask into bits: bit c of row r is set when
 *   kind 0 (int8/uint8/bool): element != 0
 *   kind 1 (fp32), 2 (fp16), 3 (bf16): element == 0   (additive float mask)
 * Element (b, r, c) is at src + b*s_b + r*s_r + c*s_c (elements).
 * out: [batch][rows][words] uint64, words = out_sr >= ceil(cols/64),
 * row stride out_sr words, batch stride out_sb words. */
int tv_pack_mask(int32_t kind, const void* src, int64_t s_b, int64_t s_r, int64_t s_c,
                 int32_t batch, int32_t rows, int32_t cols,
                 uint64_t* out, int64_t out_sb, int64_t out_sr, void* stream);

/* Per (batch, 64-key word) of a packed mask [batch][rows][words] (strides
 * sb, sr in words): out[b * out_sb + w] = 1 when word w is all ones in every
 * row, else 0.  For tv_attn_args.mask_words_full: a mask that leaves a long
 * shared prefix visible to every row (bundle verification,
 * bundle_verifier.py:166-216, masks the whole key range) then costs the
 * verify kernel nothing there.  No counterpart in the reference. */
int tv_mask_word_summary(const uint64_t* bits, int32_t batch, int32_t rows, int32_t words, int64_t sb, int64_t sr,
                         uint8_t* out, int64_t out_sb, void* stream);

/* ---- acceptance --------------------------------------------------------
 * One target token per node, then the acceptance rule of verify_new:
 *   ok[i] = draft[i] == next[parent(i)], ok[0] = 1, closure
 *   ok &= ok[parent] for min(max_depth + 2, rows) synchronous rounds,
 *   best = first argmax of (ok ? pos : 0), path = root .. best.
 * mode 0: next = argmax over the vocabulary (first maximum; NaN counts as
 *         the maximum, first NaN wins);
 * mode 1: next = sample from softmax(logits / temperature) by the Gumbel-max
 *         rule with counter-based Philox4x32-10 noise keyed by (seed, offset,
 *         row, token);
 * mode 2: next = sampled[] given by the caller.
 * parent[] has rows-1 entries: the parent's index among draft nodes, -1 for
 * children of the root (a value equal to its own index also means -1).
 *
 * result (device int64, length 8 + 2*rows):
 *   [0] status (0 ok, else TV_ERR_INPUT: parent out of range / cycle)
 *   [1] best (max_id)    [2] path length n = accept_length + 1
 *   [3] next_token       [4..7] reserved
 *   [8 .. 8+rows)        path node ids, root first
 *   [8+rows .. 8+2rows)  path draft tokens
 * next_tokens (device int64 [rows]) receives the per-node target tokens.
 * workspace: tv_accept_workspace_size() bytes. */
typedef struct tv_accept_args {
  int32_t mode;
  int32_t logits_dtype;          /* TV_BF16, TV_F16 or TV_F32               */
  const void* logits;
  int64_t logits_sm;             /* row stride (elements)                   */
  int32_t rows, vocab;
  const int64_t* draft;          /* [rows]                                  */
  const int64_t* parent;         /* [rows - 1]                              */
  const int64_t* pos;            /* [rows]                                  */
  int32_t max_depth;
  const int64_t* sampled;        /* mode 2                                  */
  float temperature;             /* mode 1                                  */
  uint64_t seed, offset;         /* mode 1                                  */
  int64_t* next_tokens;
  int64_t* result;
  void* workspace;
  size_t workspace_bytes;
} tv_accept_args;

int tv_accept_workspace_size(const tv_accept_args* args, size_t* bytes);
int tv_accept(const tv_accept_args* args, void* stream);

/* ---- compaction -------------------------------------------------------
 * Contiguous cache: for every slice s < num_slices of `data`
 * (slice base = data + s * slice_stride_bytes, row r at
 * + r * row_stride_bytes, row_bytes bytes per row) move row
 * start + path[j] to start + j for j < n, gathering all rows of a slice
 * before writing any.  path and n are read from an accept result buffer on
 * the device (n <= max_rows). */
int tv_compact_contig(void* data, int64_t num_slices, int64_t slice_stride_bytes,
                      int64_t row_stride_bytes, int32_t row_bytes, int64_t start,
                      const int64_t* accept_result, int32_t max_rows, void* stream);

/* Paged pool copy-on-write: copy whole pages src -> dst for every plane
 * (plane = layer x K/V) and head.  pairs: device int32 [npairs][2] (src, dst).
 * Page p of plane l starts at pool + l * plane_stride_bytes
 * + p * page_stride_bytes; page_bytes contiguous bytes per page. */
int tv_copy_pages(void* pool, int32_t planes, int64_t plane_stride_bytes,
                  int64_t page_stride_bytes, int64_t page_bytes,
                  const int32_t* pairs, int32_t npairs, int32_t num_pages, void* stream);

/* Paged compaction: move logical row start + path[j] to start + j for every
 * plane and head.  Sources are read through `src_table` (logical page ->
 * physical page before the move), destinations written through `dst_table`
 * (after the caller's copy-on-write remap; run tv_copy_pages first).  Both
 * are device int32 [table_len].  Row (plane l, page p, head h, offset o)
 * starts at pool + l*plane_stride_bytes + p*page_stride_bytes
 * + h*head_stride_bytes + o*row_stride_bytes.  A negative page id reads as
 * zeros and is never written. */
int tv_compact_paged(void* pool, int32_t planes, int32_t heads, int64_t plane_stride_bytes,
                     int64_t page_stride_bytes, int64_t head_stride_bytes,
                     int64_t row_stride_bytes, int32_t row_bytes, int32_t page_size,
                     const int32_t* src_table, const int32_t* dst_table, int32_t table_len,
                     int32_t num_pages, int64_t start, const int64_t* accept_result,
                     int32_t max_rows, void* stream);

/* Chunk arena gather: for every copy (chunk c, arena slot o), layer l, K/V
 * and head h, copy rows [c*chunk, min((c+1)*chunk, src_len)) of the source
 * layer cache into arena rows [o*chunk, ...).
 *   src_k / src_v: device uint64 [layers] base pointers of [heads][src_len] rows
 *   (head stride src_head_stride_bytes, row stride src_row_stride_bytes);
 *   arena row (l, kv, h, r) at arena + l*arena_layer_stride_bytes
 *   + kv*arena_kv_stride_bytes + h*arena_head_stride_bytes + r*row_bytes.
 * copies: device int32 [ncopies][2]. */
int tv_arena_gather(int32_t layers, int32_t heads, const uint64_t* src_k, const uint64_t* src_v,
                    int64_t src_head_stride_bytes, int64_t src_row_stride_bytes, int32_t src_len,
                    void* arena, int64_t arena_layer_stride_bytes, int64_t arena_kv_stride_bytes,
                    int64_t arena_head_stride_bytes, int32_t row_bytes, int32_t chunk_size,
                    int32_t arena_rows, const int32_t* copies, int32_t ncopies, void* stream);

/* Zero-copy arena: out[i * pages_per_chunk + j] =
 *   page_table[chunk_ids[i] * pages_per_chunk + j] for i < nchunks. */
int tv_gather_page_table(const int32_t* page_table, int32_t table_len, const int32_t* chunk_ids,
                         int32_t nchunks, int32_t pages_per_chunk, int32_t* out, void* stream);

/* ---- rotary embedding + KV append -------------------------------------------
 * Replaces the step before the verify attention in LlamaAttention.forward
 * (llama_target_model.py:765-783): rotate_half RoPE of q and k
 * (apply_rotary_pos_emb :429-449, apply_rotary_pos_emb_L31 :452-474) and
 * KVCache.cat of the rotated k and of v (cache_state.py:52-66), one launch.
 *
 * Tensors are [B, heads, T, D] with any strides (element units) and unit
 * stride on D; D even, D <= 256.  dtype covers q, k, v, cos, sin, the outputs
 * and the caches.  Output element (b, h, t, d) of q (and k):
 *   R(R(x[d] * cos[d]) + R(rot(x)[d] * sin[d])),  rot(x) = cat(-x2, x1),
 * R = rounding to dtype after every product and the sum, as the reference's
 * torch element-wise ops do (fp32: no fused multiply-add).  cos / sin element
 * (b, t, d) is read at cos[b * cs_sb + row * cs_sr + d] with row =
 * pos[b * pos_sb + t] when pos is given (the cached table gathered by
 * position ids) or row = t (per-token tables, as LlamaRotaryEmbedding_L31
 * returns them).  q_out may alias q.  k_out (optional) receives rotated k.
 * Cache append (optional, k_cache / v_cache): token t of batch b goes to
 * token index start + t of the cache:
 *   page_table == NULL: contiguous [B, kv_heads, capacity, D] with strides
 *     (kc_sb, kc_sh, kc_st) / (vc_sb, vc_sh, vc_st);
 *   page_table != NULL: paged pool [num_pages, kv_heads, page_size, D], page
 *     id page_table[b * pt_sb + idx / page_size], strides (kc_sb = page,
 *     kc_sh = head, kc_st = token) and the same for v.
 * A position row outside [0, cs_rows), a token index past capacity or a page
 * id outside [0, num_pages) skips that token and sets *status (if given) to
 * TV_ERR_INPUT. */
typedef struct tv_rope_args {
  int32_t dtype;                  /* TV_BF16, TV_F16 or TV_F32              */
  int32_t batch, tokens, heads, kv_heads, head_dim;
  const void* q;
  int64_t q_sb, q_sh, q_st;
  const void* k;
  int64_t k_sb, k_sh, k_st;
  const void* v;                  /* may be NULL when nothing is appended    */
  int64_t v_sb, v_sh, v_st;
  const void* cos;
  const void* sin;
  int64_t cs_sb, cs_sr, cs_rows;
  const int64_t* pos;             /* NULL: row = t                           */
  int64_t pos_sb;
  void* q_out;                    /* required                                */
  int64_t qo_sb, qo_sh, qo_st;
  void* k_out;                    /* NULL: rotated k only goes to the cache  */
  int64_t ko_sb, ko_sh, ko_st;
  void* k_cache;                  /* NULL: no append                         */
  int64_t kc_sb, kc_sh, kc_st;
  void* v_cache;
  int64_t vc_sb, vc_sh, vc_st;
  int64_t start, capacity;
  const int32_t* page_table;
  int64_t pt_sb;
  int32_t page_size, num_pages;
  int32_t* status;                /* optional device word                    */
} tv_rope_args;

int tv_rope_append(const tv_rope_args* args, void* stream);

/* ---- lm_head + acceptance ----------------------------------------------------
 * Replaces the step after the verify attention: logits = lm_head(hidden)
 * (diffspec_model.py:229-231, a [rows, vocab] tensor) followed by the argmax
 * or sampling of verify_new (tree_verification.py:100-162).  One tensor-core
 * GEMM streams the weight once and reduces every row's logits in its
 * epilogue, so the logits are never written; then the acceptance rule of
 * tv_accept runs on the per-row picks.
 *   x [rows, hidden] (row stride x_sm), weight [vocab, hidden] (row stride
 *   w_sv), dtype TV_BF16 or TV_F16 for both; rows <= 128; hidden a
 *   multiple of 64; 16-byte aligned rows.
 * Each logit is the fp32 dot product rounded to dtype (the reference's lm_head
 * returns dtype logits); mode 0 takes the argmax (ties: smaller index, a NaN
 * beats every number), mode 1 the argmax of logit / temperature + Gumbel noise
 * (the same noise as tv_accept mode 1 for the same seed / offset).
 * draft / parent / pos / max_depth / result as tv_accept; draft == NULL
 * computes next_tokens only.  workspace: tv_lmhead_accept_workspace_size. */
typedef struct tv_lmhead_args {
  int32_t dtype;
  int32_t rows, hidden, vocab;
  const void* x;
  int64_t x_sm;
  const void* weight;
  int64_t w_sv;
  int32_t mode;
  float temperature;
  uint64_t seed, offset;
  const int64_t* draft;
  const int64_t* parent;
  const int64_t* pos;
  int32_t max_depth;
  int64_t* next_tokens;
  int64_t* result;
  void* workspace;
  size_t workspace_bytes;
} tv_lmhead_args;

int tv_lmhead_accept_workspace_size(const tv_lmhead_args* args, size_t* bytes);
int tv_lmhead_accept(const tv_lmhead_args* args, void* stream);

/* ---- final draft-tree build ---------------------------------------------------
 * Replaces DraftTree.update's final branch and generate_attention_mask
 * (runtime/draft_tree.py:188-260) -- the reference walks the ancestors with a
 * host sync per hop -- plus the root row / column the verify step prepends
 * (diffspec_model.py:620-624).  One CTA:
 *   top_index [k] int64: the running top-k linear indices depth * nnodes + col;
 *   parents_matrix / input_ids_matrix [>= depth, nnodes] int64 (row strides);
 *   d2t [d2t_len] (optional): token = id + d2t[id] (draft -> target vocabulary).
 * Nodes are ordered by depth, keeping the top-k order among equal depths.
 * Outputs ([k] int64): input_ids, position_ids (= depth + 1), parent_pos (-1:
 * none); mask (optional) [k, k] int8 self + ancestors (at most depth - 1
 * hops); mask_bits (optional) [k + 1, ceil((k + 1) / 64)] uint64, the verify
 * bitmask with the root prepended (root row: itself; root column: all).
 * A top index outside [0, depth * nnodes), a repeated index or an id outside
 * d2t sets *status (if given) to TV_ERR_INPUT. */
/* ---- draft-side chunk retrieval ------------------------------------------------
 * Replaces the retrieval branch of DraftNetwork._select_working_cache_from_chunks
 * (draft/draft_network.py:1514-1612; no semantic penalty).
 * tv_chunk_select (one CTA): chunk score = (attention summed over the chunk,
 *   prefix indices clamped to attn_len as the reference's prefix sums are) /
 *   max(end - start, 1); the top_k best (NaN largest, ties to the smaller id)
 *   in ascending id order into selected[top_k]; the union of their
 *   [start, end) intervals clamped to [0, length] as ascending token indices
 *   into indices[max_indices], their number into *count.  nchunks <= 2048,
 *   top_k <= 1024.  More than max_indices indices, or a chunk bound < 0, sets
 *   *status to TV_ERR_INPUT (then nothing is written past max_indices).
 *   workspace: tv_chunk_select_workspace_size bytes (per-chunk sums).
 * tv_gather_rows: for every plane p < planes (src[p], dst[p]: device
 *   pointers, e.g. each layer's K and V), every head h < heads and every
 *   i < *count (at most max_rows): copy row_bytes from src[p] + h *
 *   src_head_stride_bytes + indices[i] * src_row_stride_bytes to dst[p] + h *
 *   dst_head_stride_bytes + i * dst_row_stride_bytes.  row_bytes a multiple
 *   of 16, 16-byte aligned rows. */
int tv_chunk_select_workspace_size(int32_t nchunks, int64_t attn_len, size_t* bytes);
int tv_chunk_select(const float* attn, int64_t attn_len, const int64_t* starts, const int64_t* ends,
                    int32_t nchunks, int32_t top_k, int64_t length, int64_t* selected, int64_t* indices,
                    int64_t max_indices, int64_t* count, void* workspace, size_t workspace_bytes,
                    int32_t* status, void* stream);
int tv_gather_rows(int32_t planes, int32_t heads, const uint64_t* src, const uint64_t* dst,
                   int64_t src_head_stride_bytes, int64_t src_row_stride_bytes, int64_t dst_head_stride_bytes,
                   int64_t dst_row_stride_bytes, int32_t row_bytes, const int64_t* indices, const int64_t* count,
                   int64_t max_rows, void* stream);

int tv_tree_finalize(int32_t nnodes, int32_t depth, int32_t k, const int64_t* top_index,
                     const int64_t* parents_matrix, int64_t pm_stride, const int64_t* input_ids_matrix,
                     int64_t im_stride, const int64_t* d2t, int64_t d2t_len, int64_t* input_ids,
                     int64_t* position_ids, int64_t* parent_pos, int8_t* mask, uint64_t* mask_bits,
                     int32_t* status, void* stream);

/* ---- decoder-layer elementwise work around the verify path --------------------
 * tv_rms_norm replaces LlamaRMSNorm.forward (runtime/llama_target_model.py:124-138):
 *   y[r] = weight * T(x[r] * rsqrt(mean(x[r]^2) + eps)), statistics in fp32,
 *   the normalised row rounded to T before the weight multiply.
 * tv_silu_mul replaces act_fn(gate_proj(x)) * up_proj(x) of LlamaMLP.forward
 *   (:506-538, act_fn = SiLU): out[r] = T(silu(gate[r])) * up[r].
 * Strides in elements; cols a multiple of 8; pointers 16-byte aligned and
 * strides multiples of 8 elements (TV_ERR_ALIGN otherwise). */
int tv_rms_norm(const void* x, int64_t x_row_stride, const void* weight, void* y, int64_t y_row_stride,
                int32_t rows, int32_t cols, float eps, int32_t dtype, void* stream);
int tv_silu_mul(const void* gate, const void* up, int64_t in_row_stride, void* out, int64_t out_row_stride,
                int32_t rows, int32_t cols, int32_t dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPECVERIFY_H_ */
