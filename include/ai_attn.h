/*
 * ai_attn.h - C ABI of the B200 chain-of-edits (multi-segment RoPE) causal
 * attention, forward and backward.
 *
 * The reference (AutodeskAILab/autoindexer, package
 * src/autoindexer/models/autoindexer) has no native FFI: its backends are
 * Python functions registered into transformers' ALL_ATTENTION_FUNCTIONS.  The
 * entry points below replace the compute those backends perform:
 *
 *   ai_attn_fwd  <- attention/triton_wrapper.py:57-101 fused_chain_of_edits_attn_triton
 *                   (-> kernels/triton_rope_attn.py:1710-1812 FusedMultiSegmentRoPEAttn.forward)
 *                   and attention/cutedsl/wrapper.py:127-170 fused_chain_of_edits_attn_cutedsl;
 *                   numerics of attention/reference.py:116-141 chain_of_edits_attn_ref.
 *   ai_attn_bwd  <- kernels/triton_rope_attn.py:1814-1902 FusedMultiSegmentRoPEAttn.backward
 *                   (and the CuTeDSL path's FA4 backward + PrepPackBackward +
 *                   FastRopeKeyFunction.backward, cutedsl/prep_multi_head/autograd.py:22-69).
 *   AiAttnLayout <- the PositionBlockList arrays the backends read
 *                   (perturb_labels.py:341-357 concat(): boundary_indices,
 *                   concat_key_pos_ids, concat_attn_masks, concat_abs_pos_masks,
 *                   query_pos_ids) plus the rotary cos/sin the RotaryEmbeddingFunc
 *                   produces (perturb_labels.py:333-339 get_rotary_pos_emb).
 *
 * Conventions
 *   - Every pointer is a device pointer unless stated otherwise.  The caller
 *     allocates every buffer (the backward's scratch through
 *     ai_attn_bwd_workspace); the library never allocates device memory.
 *   - A 4-D tensor (B, H, T, D) is described by AiTensor4: element strides of
 *     the b, h and t dimensions; the d dimension is contiguous.
 *   - All launches go on the given stream (a cudaStream_t passed as void*).
 *   - Return value: 0 = success; > 0 = the arguments were rejected on the host
 *     and nothing was launched; the text is available from ai_attn_strerror.
 *     Kernels never trap: a device-side failure (bounded wait expired, an index
 *     out of range) is written as a negative code into *status (if status is
 *     not NULL) and can be read back with ai_attn_read_status.
 */
#ifndef AI_ATTN_H
#define AI_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AI_ATTN_ABI_VERSION 9

typedef enum AiDtype {
  AI_DTYPE_BF16 = 0,
  AI_DTYPE_F16 = 1,
  AI_DTYPE_F32 = 2
} AiDtype;

enum AiStatus {
  AI_OK = 0,
  AI_ERR_NULL = 1,        /* a required pointer is NULL */
  AI_ERR_SHAPE = 2,       /* batch/seq/heads inconsistent (Hq % Hkv, sizes <= 0) */
  AI_ERR_HEAD_DIM = 3,    /* head_dim not 32, 64 or 128 */
  AI_ERR_DTYPE = 4,       /* dtype not supported */
  AI_ERR_STRIDE = 5,      /* a stride is negative or not 16-byte compatible */
  AI_ERR_ALIGN = 6,       /* a base pointer is not 16-byte aligned */
  AI_ERR_LAYOUT = 7,      /* block table / work list inconsistent with the call */
  AI_ERR_WORKSPACE = 8,   /* workspace missing or too small */
  AI_ERR_LAUNCH = 9,      /* a CUDA launch failed (the CUDA error is not cleared) */
  AI_ERR_NO_DEVICE = 10,  /* current device is not an sm_100 part */
  AI_ERR_TMA = 11,        /* tensor map encoding refused the tensor */
  AI_ERR_NOALLOC_LIMIT = 12, /* batch * num_q_heads * seq_len > AI_ATTN_NOALLOC_MAX_ROWS */
  AI_ERR_DEV_TIMEOUT = -1, /* device: a bounded wait expired */
  AI_ERR_DEV_BOUNDS = -2   /* device: an index fell outside its table */
};

/* (B, H, T, D) view: element (b, h, t, d) is at ptr[b*stride_b + h*stride_h + t*stride_t + d]. */
typedef struct AiTensor4 {
  void* ptr;
  int64_t stride_b;
  int64_t stride_h;
  int64_t stride_t;
} AiTensor4;

/* Block record, int32[8] per block (AI_BLOCK_* index the fields). */
#define AI_BLOCK_ROW 0     /* batch row the block belongs to */
#define AI_BLOCK_START 1   /* first query row s */
#define AI_BLOCK_END 2     /* one past the last query row e; keys are [0, e) */
#define AI_BLOCK_KEY_OFF 3 /* offset of key 0 of this block in key_info */
#define AI_BLOCK_KV_LO 4   /* first key with attn_mask set (e if none) */
#define AI_BLOCK_FLAGS 5   /* AI_BLOCKF_* */
#define AI_BLOCK_ABS_LO 6  /* blocks with AI_BLOCKF_ABS: first key with abs_pos_mask (and attn_mask) set */
#define AI_BLOCK_ABS_HI 7  /* ... one past the last such key; ABS_HI <= ABS_LO means "any key of the block"
                              (ABI 7: key tiles outside [ABS_LO, ABS_HI) take the fast kernels) */
#define AI_BLOCK_FIELDS 8
#define AI_ROT_CLASS_KEYS 64 /* keys per rotation-class chunk (AiAttnLayout.chunk_cls) */
#define AI_BLOCKF_MASKED 1 /* some key in [kv_lo, e) has attn_mask false */
#define AI_BLOCKF_ABS 2    /* some key has abs_pos_mask set */
#define AI_BLOCKF_OWNPOS 4 /* every attended key has the position k_own gives it (so a K copy
                              rotated once per key serves this block) */

/* key_info word: bits 0..29 rotary table row, bit 30 attn_mask, bit 31 abs_pos_mask. */
#define AI_KEY_ROW_MASK 0x3FFFFFFF
#define AI_KEY_ATTN 0x40000000u
#define AI_KEY_ABS 0x80000000u

typedef struct AiAttnLayout {
  int32_t n_blocks;
  const int32_t* blocks;      /* [n_blocks][AI_BLOCK_FIELDS], grouped by batch row */
  const int32_t* row_blocks;  /* [B + 1]: blocks of row b are [row_blocks[b], row_blocks[b+1]) */
  const int32_t* row_cov;     /* [B]: rows >= row_cov[b] belong to no block (diagonal-only) */
  const int32_t* key_info;    /* [n_keys] */
  int64_t n_keys;
  const int32_t* q_pos;       /* [B][T] rotary table row of each query row */
  const int32_t* k_own;       /* [B][T] rotary table row of key j in the block whose query rows hold j */
  const float* rope_cos;      /* [n_pos][D/2] fp32: cos of the angle of (table row, frequency slot) */
  const float* rope_sin;      /* [n_pos][D/2] */
  const void* rope_cs16;      /* [n_pos][D/2] fp16 pairs (cos, sin) of the same angles: the bf16 kernels'
                                 copy (fp16 keeps 11 bits, above the bf16 operands they rotate) */
  int32_t n_pos;
  int32_t fwd_tile;           /* query rows per forward / dQ work item (ai_attn_fwd_tile_rows) */
  const int32_t* fwd_items;   /* [n_fwd_items][4]: block, q0, q1, 0 */
  int32_t n_fwd_items;
  int32_t n_fwd_abs_items;    /* the first n_fwd_abs_items items belong to blocks with AI_BLOCKF_ABS */
  int32_t kv_tile;            /* keys per dK/dV work item (ai_attn_kv_tile_rows) */
  const int32_t* kv_items;    /* [n_kv_items][4]: row, j0, j1, 0 */
  int32_t n_kv_items;
  int32_t n_kv_abs_items;     /* the first n_kv_abs_items items hold an abs key of some block */
  int32_t all_rows_owned;     /* 1: row_cov[b] == seq_len for every b (no diagonal-only rows), so the
                                 fill launches are skipped; 0: not known (they run) */
  int32_t n_fwd_short_items;  /* the n_fwd_short_items items right after the abs items have at most
                                 fwd_tile / 2 query rows (ABI 7): with four or more query heads per KV
                                 head the tensor-core kernels pack two heads' rows of such an item into
                                 one 128-row tile; 0: no item is treated as short */
  /* dK/dV work split (ABI 8; all optional: n_kv_chunks = 0 runs one CTA per key tile).  The 64-row
     query tiles a key tile's blocks give it (blocks with an abs key among its keys left out) are
     numbered in block order; a chunk is a range of them.  A key tile with one chunk is written
     directly; the chunks of a longer one write fp32 partial sums (ai_attn_bwd_workspace counts
     them) that one more launch adds up in chunk order (deterministic). */
  const int32_t* kv_chunks;   /* [n_kv_chunks][4]: kv item, first query tile, end query tile, partial
                                 slot (-1: the item's only chunk) */
  int32_t n_kv_chunks;
  int32_t n_kv_partials;      /* partial slots */
  const int32_t* kv_reduce;   /* [n_kv_reduce][4]: kv item, first slot, slots, 0 */
  int32_t n_kv_reduce;
  int32_t kv_cost_max;        /* work of the costliest key tile and of all key tiles (query tiles
                                 plus two per block a key tile walks): the chunks run only when the
                                 costliest tile outweighs the average work of an SM */
  int32_t kv_cost_total;
  /* Rotation classes (ABI 9; optional: n_rot_classes = 0 turns them off).  The keys of a block
     without AI_BLOCKF_OWNPOS whose kv_lo is a multiple of 64 are taken in 64-key chunks
     [kv_lo + 64 i, kv_lo + 64 i + 64), 2 * ceil((e - kv_lo) / 128) of them (chunks past e pad the
     last 128-key tile).  Chunks of one batch row that give every attended key the same rotary
     table row, and leave the same keys unattended or past their block's end, share a class.
     When the forward workspace holds the rotated copies (ai_attn_fwd_workspace counts the
     classes) each class's chunk is rotated once per KV head, and the tensor-core kernels read it
     instead of rotating the chunk's keys in shared memory for every block that sees them. */
  const int32_t* blk_cls;     /* [n_blocks]: index in chunk_cls of the block's chunk 0, -1: no classes */
  const int32_t* chunk_cls;   /* [n_chunk_cls]: class of each chunk */
  int32_t n_chunk_cls;
  const int32_t* rot_classes; /* [n_rot_classes][2]: block and first key of a chunk with the class's rows */
  int32_t n_rot_classes;
  int32_t n_fwd_abs_short_items; /* the first n_fwd_abs_short_items of the abs items have at most
                                    fwd_tile / 2 rows (ABI 9); with the split below they pack four heads
                                    of a GQA group per unit on the persistent kernels */
} AiAttnLayout;

typedef struct AiAttnFwdArgs {
  int32_t batch;
  int32_t seq_len;
  int32_t num_q_heads;
  int32_t num_kv_heads;   /* GQA: num_q_heads % num_kv_heads == 0; no expanded copy of K/V */
  int32_t head_dim;
  int32_t dtype;          /* AiDtype of q, k, v, out */
  float scale;            /* softmax scale applied to the logits */
  AiTensor4 q;            /* (B, Hq, T, D) */
  AiTensor4 k;            /* (B, Hkv, T, D) */
  AiTensor4 v;            /* (B, Hkv, T, D) */
  AiTensor4 out;          /* (B, Hq, T, D) view of the (B, T, Hq, D) output */
  float* lse;             /* (B, Hq, T) natural-log log-sum-exp of the scaled logits */
  AiAttnLayout layout;
  int32_t* status;        /* optional device status word */
  void* workspace;        /* optional scratch (256-B aligned); with ai_attn_fwd_workspace bytes the
                             tensor-core kernels read once-rotated copies of Q and K from it, with
                             less (or NULL) they rotate every tile in shared memory */
  size_t workspace_bytes;
} AiAttnFwdArgs;

typedef struct AiAttnBwdArgs {
  AiAttnFwdArgs fwd;      /* the forward's arguments; out and lse as the forward wrote them */
  AiTensor4 dout;         /* (B, Hq, T, D) view of dL/dout */
  AiTensor4 dq;           /* (B, Hq, T, D) */
  AiTensor4 dk;           /* (B, Hkv, T, D), summed over the query heads of each group */
  AiTensor4 dv;           /* (B, Hkv, T, D) */
  void* workspace;        /* device scratch, 256-B aligned: at least B*Hq*T floats (rounded up to
                             256 B); ai_attn_bwd_workspace bytes also hold the rotated Q/K copies */
  size_t workspace_bytes;
  int32_t fwd_rotated;    /* 1: fwd.workspace still holds the once-rotated Q/K copies that ai_attn_fwd
                             wrote for these q, k and layout (fwd.workspace_bytes >=
                             ai_attn_fwd_workspace); the backward reads them instead of rotating
                             again, and its own workspace needs only the B*Hq*T floats.
                             0: fwd.workspace is ignored. */
  int32_t parts;          /* ABI 9: 0 (or AI_BWD_DQ | AI_BWD_DKDV) runs the whole backward.
                             AI_BWD_DQ: the row sums of dO.O, the rotated copies when needed, dQ and
                             the rows no block owns; AI_BWD_DKDV: dK and dV only, reading what a
                             preceding AI_BWD_DQ call with the same arguments and workspace left
                             there (stream order).  The two calls let a caller start using dQ (an
                             all-gather, say) while dK and dV are computed.  The fp32 / fp16 path
                             computes every gradient in the AI_BWD_DQ call. */
} AiAttnBwdArgs;

#define AI_BWD_DQ 1
#define AI_BWD_DKDV 2

/* ABI version this library was built with (AI_ATTN_ABI_VERSION). */
int ai_attn_abi_version(void);

/* Query rows per forward/dQ work item, and keys per dK/dV work item, for a
 * (dtype, head_dim); the caller's work lists must be tiled with these. */
int ai_attn_fwd_tile_rows(int dtype, int head_dim);
int ai_attn_kv_tile_rows(int dtype, int head_dim);

/* Forward: out and lse for every row (rows no block owns get out = v of the
 * row and lse = 0, the reference's diagonal-only convention). */
int ai_attn_fwd(const AiAttnFwdArgs* args, void* stream);

/* Bytes of forward scratch for the fastest path (0 when the dtype / head_dim
 * has no use for it). */
int ai_attn_fwd_workspace(const AiAttnFwdArgs* args, size_t* bytes);

/* Bytes of backward scratch for the fastest path (the minimum is
 * B*Hq*T floats rounded up to 256 B). */
int ai_attn_bwd_workspace(const AiAttnBwdArgs* args, size_t* bytes);

/* Backward: dq, dk, dv (written, not accumulated). */
int ai_attn_bwd(const AiAttnBwdArgs* args, void* stream);

/* Backward for callers that cannot allocate device memory (no counterpart in
 * the reference, which allocates through PyTorch).  Same results as
 * ai_attn_bwd given a workspace of the same 16 MiB; args->workspace is
 * ignored: the scratch comes from a fixed 16 MiB array inside the library
 * (held on every GPU that loads it until the process exits), so
 * batch * num_q_heads * seq_len must not exceed AI_ATTN_NOALLOC_MAX_ROWS
 * (else AI_ERR_NOALLOC_LIMIT, nothing launched).  The array holds the row
 * sums of dO.O and, when fwd_rotated is 0 and they fit (B * Hq * T up to
 * about 50,000 at head_dim 128 with four query heads per KV head), the
 * rotated Q/K copies; larger calls rotate every tile in shared memory
 * instead (slower).  Calls no allocator.  The
 * first call on a device looks the array up on that device; make it before
 * any stream capture.  Calls that overlap on the GPU share the array and
 * race. */
#define AI_ATTN_NOALLOC_MAX_ROWS (1 << 22)
int ai_attn_bwd_noalloc(const AiAttnBwdArgs* args, void* stream);

/* Decode step: one query token per batch row against an unrotated K/V cache.
 *
 *   ai_attn_decode <- attention/__init__.py:39-51, the IterPositions branch of the registered
 *                     attention interface (keys expanded by repeat_kv, :36-37), with
 *                     attn_layers.py:15-27 compute_attn_weights_iter: each key rotated by its own
 *                     position id (IterPositions.key_pos_ids, type_utils.py:48-67), the query
 *                     unrotated, attn_mask, scale, softmax, P.V.
 *
 * The reference rotates the whole cache and expands K/V for GQA every token;
 * here every key is rotated as it is read, each KV head's cache is read once
 * for its whole query-head group, and the keys are split over CTAs whose
 * partial results a second launch combines.  bf16, head_dim 128, at most 8
 * query heads per KV head.  A row whose keys are all masked returns zeros. */
typedef struct AiAttnDecodeArgs {
  int32_t batch;
  int32_t kv_len;             /* L: keys in the cache */
  int32_t num_q_heads;
  int32_t num_kv_heads;       /* num_q_heads / num_kv_heads <= 8 */
  int32_t head_dim;           /* 128 */
  int32_t dtype;              /* AI_DTYPE_BF16 */
  float scale;                /* softmax scale applied to the logits */
  AiTensor4 q;                /* (B, Hq, 1, D) */
  AiTensor4 k;                /* (B, Hkv, L, D) unrotated cache */
  AiTensor4 v;                /* (B, Hkv, L, D) */
  AiTensor4 out;              /* (B, Hq, 1, D) */
  const int32_t* key_rows;    /* [B or 1][L]: rotary table row of each key's position id */
  int64_t key_rows_stride_b;  /* elements between rows; 0: one position row shared by the batch */
  const uint8_t* key_ok;      /* [B or 1][L]: 1 = the key is attended; NULL: every key */
  int64_t key_ok_stride_b;    /* 0: one mask row shared by the batch */
  const void* rope_cs16;      /* [n_pos][D/2] fp16 pairs (cos, sin), as AiAttnLayout.rope_cs16 */
  int32_t n_pos;
  int32_t* status;            /* optional device status word */
  void* workspace;            /* device scratch, 256-B aligned, ai_attn_decode_workspace bytes */
  size_t workspace_bytes;
} AiAttnDecodeArgs;

/* Scratch the decode step needs (the split-K partial results). */
int ai_attn_decode_workspace(const AiAttnDecodeArgs* args, size_t* bytes);

/* out = softmax(scale * q . R(pos_j) k_j masked) . v, per (row, query head). */
int ai_attn_decode(const AiAttnDecodeArgs* args, void* stream);

/* ------------------------------------------------------------------------
 * Index-head cursor attention (the edit-cursor losses of the index head).
 *
 *   ai_index_fwd / ai_index_bwd <- attn_layers.py:40-110 compute_index_losses (with
 *                                  :15-27 compute_attn_weights_iter and :30-37
 *                                  compute_end_index_mask): per edit a start row (head 0) and
 *                                  an end row (head 1), each q . R(rel_j) k_j over a key prefix,
 *                                  masked, scaled, -log_softmax at the cursor key.  The
 *                                  reference runs a Python loop of small torch ops per edit;
 *                                  here one launch runs every row (forward) and two launches
 *                                  the backward, without atomics.
 * ------------------------------------------------------------------------ */
typedef struct AiIndexArgs {
  int32_t batch;
  int32_t seq_len;
  int32_t head_dim;          /* 32, 64 or 128 */
  int32_t dtype;             /* AI_DTYPE_BF16 or AI_DTYPE_F32 (q, k, dq, dk) */
  float scale;
  AiTensor4 q;               /* (B, 2, T, D) index-head queries, unrotated */
  AiTensor4 k;               /* (B, 2, T, D) index-head keys, unrotated */
  int32_t n_rows;            /* index rows (two per edit) */
  const int32_t* rows;       /* [n_rows][4]: head, query row, n (the row sees keys [0, n)),
                                offset of its keys in key_rows / key_ok / logits */
  const int32_t* targets;    /* [n_rows]: the cursor key of the row, in [0, n) */
  int64_t n_keys;            /* entries of key_rows / key_ok (sum of n over the rows) */
  const int32_t* key_rows;   /* rotary table row of each key's position relative to the query */
  const uint8_t* key_ok;     /* 1: the key may be attended */
  const float* rope_cos;     /* [n_pos][D/2] */
  const float* rope_sin;
  int32_t n_pos;
  float* logits;             /* [B][n_keys] out: scaled logits, -inf where masked (read by the backward) */
  float* lse;                /* [B][n_rows] out: log-sum-exp of the row */
  float* loss;               /* [B][n_rows] out: lse - logit at the target (+inf if the target is masked) */
  int32_t* status;           /* optional device status word */
} AiIndexArgs;

typedef struct AiIndexBwdArgs {
  AiIndexArgs fwd;           /* as the forward ran, its outputs included */
  const float* dloss;        /* [B][n_rows]: dL/dloss */
  AiTensor4 dq;              /* (B, 2, T, D): the index rows are written, the other rows are left as they are */
  AiTensor4 dk;              /* (B, 2, T, D): every row is written */
} AiIndexBwdArgs;

int ai_index_fwd(const AiIndexArgs* args, void* stream);
int ai_index_bwd(const AiIndexBwdArgs* args, void* stream);


/* ------------------------------------------------------------------------
 * Host-side layout builders (plain host memory, no GPU, no allocation by the
 * caller's device).
 *
 *   ai_attn_positions_from_ops <- perturb_labels.py:236-275 perturb_labels_per_sequence,
 *                                 :395-467 get_parsed_positions_from_perturbations and
 *                                 :341-357 PositionBlockList.concat(): an edit chain (the
 *                                 operations sample_cursor_operations returns, in order) ->
 *                                 the concat()-ed arrays of its position-block list.
 *   ai_attn_prep               <- the device tables the backends build per layout
 *                                 (triton_rope_attn.py:1012-1055 build_multi_segment_launch_cache,
 *                                 cutedsl/meta.py:66-98 build_cutedsl_meta): concat()-ed lists ->
 *                                 the AiAttnLayout tables, written into host buffers for one
 *                                 host-to-device copy.  The rotary table for positions
 *                                 [p_min, p_max] is the caller's (it comes from its rotary module).
 * ------------------------------------------------------------------------ */
#define AI_BLOCK_TYPE_EXTEND 1
#define AI_BLOCK_TYPE_EDIT 2
#define AI_BLOCK_TYPE_COMPLETE 3

/* Sizes of the list an edit chain yields.  ops: n_ops rows of five int64
 * (num_insert, num_delete, start_rel_pos, end_rel_pos, num_extend); the first
 * must be a pure extend.  AI_ERR_LAYOUT for a chain the reference rejects. */
int ai_attn_positions_from_ops_sizes(const int64_t* ops, int32_t n_ops, int32_t* n_blocks, int64_t* n_query,
                                     int64_t* n_keys);
/* boundary [n_blocks][4] (start, end, key_start, key_end); query_pos [n_query];
 * key_pos, attn_mask, abs_mask [n_keys]; block_type [n_blocks] (AI_BLOCK_TYPE_*,
 * may be NULL). */
int ai_attn_positions_from_ops(const int64_t* ops, int32_t n_ops, int64_t* boundary, int64_t* query_pos,
                               int64_t* key_pos, uint8_t* attn_mask, uint8_t* abs_mask, int32_t* block_type);

/* One concat()-ed position-block list (perturb_labels.py:341-357), host memory. */
typedef struct AiPrepList {
  int32_t n_blocks;
  const int64_t* boundary;    /* [n_blocks][4]: start, end, key_start, key_end */
  int64_t n_query;            /* entries of query_pos: the last block's end */
  const int64_t* query_pos;
  int64_t n_keys;             /* entries of the key arrays: the last block's key_end */
  const int64_t* key_pos;
  const uint8_t* attn_mask;
  const uint8_t* abs_mask;    /* NULL: no abs keys */
} AiPrepList;

typedef struct AiPrepSizes {
  int32_t n_blocks;           /* block records over the batch */
  int32_t n_fwd_items;
  int32_t n_kv_items;
  int32_t n_kv_chunks;        /* entries of kv_chunks (at least n_kv_items) */
  int32_t n_kv_reduce;        /* entries of kv_reduce */
  int32_t n_chunk_cls;        /* entries of chunk_cls */
  int32_t n_rot_classes;      /* entries of rot_classes */
  int64_t n_keys;             /* key words (sum over the distinct lists) */
  int64_t p_min, p_max;       /* position ids the rotary table must cover (row r = position p_min + r) */
} AiPrepSizes;

/* Host buffers for ai_attn_prep, sized from AiPrepSizes; the counts and
 * flags come back in the last fields.  Copied to the device they are the
 * AiAttnLayout tables of the same names. */
typedef struct AiPrepTables {
  int32_t* blocks;            /* [n_blocks][AI_BLOCK_FIELDS] */
  int32_t* row_blocks;        /* [batch + 1] */
  int32_t* row_cov;           /* [batch] */
  int32_t* key_info;          /* [n_keys] */
  int32_t* q_pos;             /* [batch][seq_len] */
  int32_t* k_own;             /* [batch][seq_len] */
  int32_t* fwd_items;         /* [n_fwd_items][4] */
  int32_t* kv_items;          /* [n_kv_items][4] */
  int32_t* kv_chunks;         /* [n_kv_chunks][4] */
  int32_t* kv_reduce;         /* [n_kv_reduce][4] */
  int32_t* blk_cls;           /* [n_blocks] */
  int32_t* chunk_cls;         /* [n_chunk_cls] */
  int32_t* rot_classes;       /* [n_rot_classes][2] */
  int32_t n_kv_partials;
  int32_t kv_cost_max;
  int32_t kv_cost_total;
  int32_t n_fwd_abs_items;
  int32_t n_fwd_short_items;
  int32_t n_fwd_abs_short_items;
  int32_t n_kv_abs_items;
  int32_t all_rows_owned;
  int64_t pairs_per_head;     /* finite (query, key) logits of one head over the batch */
} AiPrepTables;

/* lists: n_lists distinct lists; list_of_row[b]: the list batch row b uses.
 * fwd_tile / kv_tile: ai_attn_fwd_tile_rows / ai_attn_kv_tile_rows. */
int ai_attn_prep_sizes(const AiPrepList* lists, int32_t n_lists, const int32_t* list_of_row, int32_t batch,
                       int32_t seq_len, int32_t fwd_tile, int32_t kv_tile, AiPrepSizes* sizes);
int ai_attn_prep(const AiPrepList* lists, int32_t n_lists, const int32_t* list_of_row, int32_t batch,
                 int32_t seq_len, int32_t fwd_tile, int32_t kv_tile, AiPrepTables* out);

/* Host side of the index head (no GPU): the rows of compute_index_losses
 * (attn_layers.py:56-104) for one concat()-ed list whose blocks carry
 * block_type (AI_BLOCK_TYPE_*).  Per EXTEND block, in block order, edit
 * marker ed = end - 1: the start row (head 0, query ed - 1, keys [0, ed),
 * rel = key_pos - query_pos[ed - 1]) and the end row (head 1, query ed, keys
 * [0, ed + 1), rel = key_pos - query_pos[ed]); a key may be attended when its
 * attn_mask is set and key_pos >= editable_start, for the end row also when
 * rel > 0.  ai_index_rows_sizes gives the counts and the edit markers (edits:
 * NULL or [n_rows / 2]); ai_index_rows writes the AiIndexArgs tables: rows,
 * key_rows (rel - rel_lo, clamped into the table) and key_ok, and the
 * relative positions [rel_lo, rel_hi] (0 included) the rotary table must
 * cover.  An EXTEND block of fewer than two rows is AI_ERR_LAYOUT. */
typedef struct AiIndexRowsOut {
  int32_t* rows;             /* [n_rows][4] */
  int32_t* key_rows;         /* [n_keys] */
  uint8_t* key_ok;           /* [n_keys] */
  int64_t rel_lo, rel_hi;    /* out */
} AiIndexRowsOut;
int ai_index_rows_sizes(const AiPrepList* list, const int32_t* block_type, int32_t* n_rows, int64_t* n_keys,
                        int64_t* edits);
int ai_index_rows(const AiPrepList* list, const int32_t* block_type, int64_t editable_start, AiIndexRowsOut* out);

/* Synchronises the stream, copies the device status word to *host_out and
 * resets it to AI_OK.  For tests and debugging; not needed on the hot path. */
int ai_attn_read_status(int32_t* dev_status, void* stream, int32_t* host_out);

/* Self-test of the device-side failure path (no reference counterpart): one
 * CTA waits, with the bounded mbarrier wait every kernel here uses, on a
 * barrier that nothing completes; after max_cycles SM clocks (1 ..
 * 2,000,000,000) the wait gives up and AI_ERR_DEV_TIMEOUT is recorded in
 * *status (a device pointer), as a kernel whose wait expired records it.
 * Nothing asynchronous is in flight, so no fault or hang can follow; read the
 * code back with ai_attn_read_status. */
int ai_attn_selftest_wait(int32_t* status, long long max_cycles, void* stream);

/* Static text for a status code. */
const char* ai_attn_strerror(int code);

/* Optional per-kernel timing (no reference counterpart; for benchmarks and
 * profiling).  While enabled, each kernel launch of this library is
 * bracketed by two CUDA events recorded on the launch's own stream (nothing
 * is skipped or reordered).  ai_attn_profile_enable(1) starts a fresh
 * collection, (0) stops it.  ai_attn_profile_read synchronises the recorded
 * events and writes, per kind, the summed elapsed milliseconds and the launch
 * count (arrays of AI_PROF_KINDS entries), then clears the collection.  At
 * most 4096 launches are recorded per collection.  Not for concurrent use
 * from several host threads. */
typedef enum AiProfKind {
  AI_PROF_PREROT = 0,   /* once-rotated Q/K copies */
  AI_PROF_FWD = 1,      /* tensor-core forward kernels */
  AI_PROF_FWD_FILL = 2, /* forward rows no block owns */
  AI_PROF_DELTA = 3,    /* row sums of dO.O */
  AI_PROF_DQ = 4,       /* tensor-core dQ kernels */
  AI_PROF_DKDV = 5,     /* tensor-core dK/dV kernels */
  AI_PROF_BWD_FILL = 6, /* backward rows no block owns */
  AI_PROF_SIMT = 7,     /* fp32 / fp16 / other head_dim path */
  AI_PROF_DECODE = 8,   /* decode step (split-K + combine) */
  AI_PROF_KINDS = 9
} AiProfKind;
int ai_attn_profile_enable(int on);
int ai_attn_profile_read(float* ms_by_kind, int32_t* launches_by_kind);

#ifdef __cplusplus
}
#endif

#endif /* AI_ATTN_H */
