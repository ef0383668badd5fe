/*
 * atflash_b200.h -- C ABI of the B200 (sm_100a) windowed-attention library.
 *
 * Windowed attention (ATFlash): RoPE pair r keeps its QK^T term only while the
 * query-key distance z <= w_r = k * lambda_r; softmax and P.V are unchanged.
 * With the pairs stored in wavelength-sorted order the kept pairs form a prefix
 * of the head dimension, so the window shortens the QK contraction to
 * D_eff(z) = 16 * #{i : zhi[i] >= z} dims (a 16-dim "level" per MMA K-step).
 *
 * Conventions
 *  - Every function returns 0 (ATF_OK) or a negative ATF_ERR_* code; nothing
 *    aborts, nothing synchronises the device unless its comment says so.
 *  - All tensor pointers are device pointers owned by the caller; strides are
 *    in elements and the innermost (head_dim) stride is 1.
 *  - Kernels run on the caller's stream. The library keeps no mutable global
 *    state except the lazily loaded driver entry point used to encode TMA
 *    descriptors and, for atf_decode_run_noalloc only, its scratch array and
 *    the address of that array in each CUDA context.
 *  - head_dim is 128. GQA group sizes 1..16 (1/2/3/4/7/8 are the tested ones).
 *  - Device-side waits are bounded. A wait that expires writes a non-zero code
 *    to params->error_flag (if not NULL) and the kernel returns early; read it
 *    with atf_read_error_flag() after synchronising.
 *
 * Reference interfaces each entry point replaces (paths inside the reference
 * project):
 *  atf_window_*      atflash/window_table.py:38-128, window_tables/atflash_window.py:52-116,
 *                    kernels/flashinfer_port/fiwin_common.py:35-60
 *  atf_prefill_fwd   the windowed FA4 forward, called as
 *                    _flash_attn_fwd(q, k, v, causal=True, pack_gqa=..., atflash_window_zhi=zhi)
 *                    at e2e_pipeline/atflash_e2e_fafi.py:119 and microbench/b1_correctness.py:84-85
 *  atf_decode_plan / atf_decode_run
 *                    the windowed FlashInfer decode, called as
 *                    single_decode_with_kv_cache_with_jit_module(mod, q, k, v, None, zhi8, ...)
 *                    at e2e_pipeline/atflash_e2e_fafi.py:106-110 (kernel diff:
 *                    kernels/flashinfer_port/decode.cuh.diff:51-89); batched and paged here
 *  atf_lse_merge     the split-KV state merge inside that FlashInfer decode
 *                    (kernels/flashinfer_port/decode.cuh.diff:62 kv_chunk_size)
 *  atf_rope_pack     the HF RoPE + sorted-pair permutation the harness applies before the
 *                    kernels (e2e_pipeline/atflash_e2e_fafi.py:186-194,
 *                    microbench/b1_correctness.py:113-135)
 */
#ifndef ATFLASH_B200_H_
#define ATFLASH_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* atf_stream_t; /* identical to cudaStream_t */

enum {
  ATF_OK = 0,
  ATF_ERR_INVALID_ARG = -1,  /* null pointer, bad shape, bad stride */
  ATF_ERR_UNSUPPORTED = -2,  /* valid but unsupported (head_dim, group size, ...) */
  ATF_ERR_ALIGNMENT = -3,    /* pointer or stride not 16-byte aligned */
  ATF_ERR_CUDA = -4,         /* a CUDA runtime / driver call failed */
  ATF_ERR_WORKSPACE = -5,    /* workspace or plan buffer too small */
  ATF_ERR_DEVICE = -6,       /* device is not sm_100 */
  ATF_ERR_TIMEOUT = -7       /* value written to error_flag by an expired device wait */
};

enum { ATF_LAYOUT_SORTED_PAIR = 0, ATF_LAYOUT_ROTATE_HALF = 1 };
enum { ATF_KV_NHD = 0, ATF_KV_HND = 1 };
enum { ATF_WINDOW_OFF = 0, ATF_WINDOW_SNAP16 = 1, ATF_WINDOW_VEC8 = 2 };
enum { ATF_DTYPE_BF16 = 0, ATF_DTYPE_F32 = 1 };

#define ATF_HEAD_DIM 128
#define ATF_MAX_LEVELS 8  /* head_dim / 16 */
#define ATF_MAX_SLICES 16 /* head_dim / 8  */

/* ------------------------------------------------------------------ tables */

/* fp32 window width of every sorted pair j: k * 2pi * base^(2(P-1-j)/d),
 * computed in fp64 and rounded to fp32; k_ret = +inf gives +inf. Writes d/2
 * floats. Replaces atflash/window_table.py:38-54. */
int atf_window_widths(int head_dim, double rope_base, double k_ret, float* wvec_out);

/* zhi[i] = max{z >= 0 : D_eff(z) >= 16(i+1)}, capped at n_ctx (d/16 entries).
 * wvec holds d/2 widths in any order. Replaces window_tables/atflash_window.py:85-116. */
int atf_window_zhi16(const float* wvec, int head_dim, int64_t n_ctx, int32_t* zhi_out);

/* vec8 slice table: zhi8[tx] = floor(w[4 tx]) (INT32_MAX for inf), d/8 entries.
 * Replaces kernels/flashinfer_port/fiwin_common.py:35-46. */
int atf_window_zhi8(const float* wvec, int head_dim, int32_t* zhi_out);

/* D_eff (dims) at distance z from a 16-snap zhi table. Replaces
 * atflash/window_table.py:62-67 evaluated through the zhi levels. */
int atf_window_deff(const int32_t* zhi16, int n_levels, int64_t z);

/* ------------------------------------------------------------------ prefill */

typedef struct {
  const void* q; /* bf16 [B, Sq, Hq, 128] (BSHD; strides below) */
  const void* k; /* bf16 [B, Sk, Hkv, 128] */
  const void* v; /* bf16 [B, Sk, Hkv, 128] */
  void* out;     /* bf16 [B, Sq, Hq, 128] */
  float* lse;    /* optional fp32 [B, Hq, Sq], natural log of sum(exp(scale*s)) */
  int64_t batch, seqlen_q, seqlen_k, num_heads_q, num_heads_kv, head_dim;
  int64_t q_stride_b, q_stride_s, q_stride_h;
  int64_t k_stride_b, k_stride_s, k_stride_h;
  int64_t v_stride_b, v_stride_s, v_stride_h;
  int64_t o_stride_b, o_stride_s, o_stride_h;
  int64_t q_offset;    /* global position of query row 0; keys are at 0..Sk-1.
                          Causal masking keeps key n for row i iff n <= q_offset + i. */
  float softmax_scale; /* usually 1/sqrt(head_dim) */
  int causal;
  int qk_layout;       /* ATF_LAYOUT_*: pair order of q and k along head_dim */
  int window;          /* ATF_WINDOW_OFF or ATF_WINDOW_SNAP16 */
  int32_t zhi[ATF_MAX_LEVELS]; /* 16-snap levels; zhi[0] must cover every distance */
  int* error_flag;     /* optional device int (see header comment) */
  /* RoPE of q at load (optional): with q_cos / q_sin given, q is the PRE-RoPE
   * query in HF rotate_half order; each query row is rotated at position
   * q_offset + row in fp32 (x1*cos - x2*sin, x2*cos + x1*sin, separately rounded
   * products), rounded to bf16 and placed in sorted-pair order as the kernel
   * loads it. k must then be post-RoPE in sorted-pair order (qk_layout). The
   * tables are fp32 [q_n_pos, >= 64]; row p holds cos / sin(p * inv_freq). */
  const float* q_cos;
  const float* q_sin;
  int64_t q_cs_stride_pos; /* elements between the tables' rows */
  int64_t q_n_pos;         /* rows in the tables; q_offset + seqlen_q <= q_n_pos */
  /* Row ranges (optional): with num_row_ranges = 1 or 2, only the query rows
   * [row_begin[i], row_end[i]) are computed, in one launch; the other rows of
   * out (and lse) are neither read nor written. A rank of a zig-zag sharded
   * prefill passes its two blocks here. Ranges are sorted, disjoint, inside
   * [0, seqlen_q), and begin on multiples of 128 (the query tile, so the window's
   * tile quantisation is the single run's). 0: every row. */
  int32_t num_row_ranges;
  int64_t row_begin[2];
  int64_t row_end[2];
} AtfPrefillParams;

/* Windowed causal prefill on the tcgen05/TMEM kernel. Tiles are 128 queries x
 * 128 keys; the window is quantised per (q-tile, k-tile) at the tile's smallest
 * distance, as atflash/reference.py:27-80 with block_m = block_n = 128. With
 * q_cos / q_sin the RoPE of q is applied at load (the RoPE front-end of
 * microbench/b1_correctness.py:113-135 for q, fused into the kernel). */
int atf_prefill_fwd(const AtfPrefillParams* p, atf_stream_t stream);

/* ------------------------------------------------------------------ decode */

typedef struct {
  int32_t batch_size;
  int32_t num_qo_heads, num_kv_heads, head_dim, page_size;
  const int32_t* indptr_host;        /* [batch+1] page ranges per request (host) */
  const int32_t* last_page_len_host; /* [batch] (host) */
  int32_t num_sms;        /* 0: query the current device */
  int32_t min_chunk_keys; /* 0: default (256) */
  int32_t max_chunk_keys; /* 0: unlimited; forces at least ceil(len/max) splits */
  /* Optional window of the run (ATF_WINDOW_SNAP16 with its zhi16 table): the
   * items are then cut to equal bytes read (V rows plus in-window K levels)
   * instead of equal key counts. OFF / VEC8: equal key counts. q_pos_host and
   * kv_pos0_host (optional, [batch], host) give the positions the run will use
   * (defaults kv_len-1 and 0); they only steer the balance, never the result. */
  int32_t window;
  int32_t zhi16[ATF_MAX_LEVELS];
  const int64_t* q_pos_host;
  const int64_t* kv_pos0_host;
} AtfDecodePlanParams;

typedef struct {
  int32_t num_items;       /* work items (request, key range) */
  int32_t chunk_keys;      /* keys of the longest item */
  int64_t partial_o_floats;   /* workspace floats needed for partial outputs */
  int64_t partial_lse_floats; /* workspace floats needed for partial LSEs */
} AtfDecodePlan;

/* Build the split-KV schedule on the host. items_host receives num_items rows
 * of int32[4] = {request, key_begin, key_end, 0}; item_indptr_host receives
 * batch+1 offsets. Pass NULL buffers to query sizes only. Items start on
 * multiples of 64 keys and hold at most 16384 keys (atf_decode_run's kernels
 * report longer or unaligned items through error_flag and skip them). */
int atf_decode_plan(const AtfDecodePlanParams* p, int32_t* items_host, int32_t items_capacity,
                    int32_t* item_indptr_host, AtfDecodePlan* out);

typedef struct {
  const void* q; /* bf16 [B, Hq, 128] */
  int64_t q_stride_b, q_stride_h;
  const void* k_cache; /* bf16 pages: NHD [P, page, Hkv, 128] or HND [P, Hkv, page, 128] */
  const void* v_cache;
  int64_t num_pages;    /* pages in the cache (page indices must be < num_pages) */
  int64_t kv_stride_page, kv_stride_token, kv_stride_head; /* same for k and v */
  int kv_layout;        /* ATF_KV_* (informational; strides carry the layout) */
  int qk_layout;        /* pair order of q and the cached k */
  const int32_t* indptr;        /* device [B+1] */
  const int32_t* indices;       /* device [nnz_pages] */
  const int32_t* last_page_len; /* device [B] */
  const int32_t* items;         /* device, from atf_decode_plan */
  const int32_t* item_indptr;   /* device [B+1], from atf_decode_plan (last entry = num_items) */
  int32_t num_items;
  int32_t batch_size, num_qo_heads, num_kv_heads, head_dim, page_size;
  const int64_t* q_pos;   /* optional device [B]: global position of the query (default kv_len-1) */
  const int64_t* kv_pos0; /* optional device [B]: global position of local key 0 (default 0) */
  float sm_scale;
  int window;                          /* ATF_WINDOW_OFF / SNAP16 / VEC8 */
  int32_t zhi16[ATF_MAX_LEVELS];       /* SNAP16: per-key 16-dim levels */
  int32_t zhi8[ATF_MAX_SLICES];        /* VEC8: per 8-dim slice (sorted-pair layout only) */
  float* partial_o;   /* workspace [num_items, Hq, 128] fp32, 16-byte aligned */
  float* partial_lse; /* workspace [num_items, Hq] fp32 (log2 domain) */
  void* out;          /* [B, Hq, 128], bf16 or fp32 per out_dtype; 8-byte aligned
                         (16 for fp32) */
  int64_t o_stride_b, o_stride_h; /* multiples of 4 elements */
  int out_dtype;      /* ATF_DTYPE_BF16 or ATF_DTYPE_F32 */
  float* lse_out;     /* optional fp32 [B, Hq], natural log */
  int* error_flag;
  /* Level-major K pages (optional, 0 = k_cache uses the kv strides above):
   * k_cache is [P, Hkv, 8 levels, page, 16] bf16 in sorted-pair order, so the
   * in-window levels of a page are one contiguous run. Needs the sorted-pair
   * layout, a page size of 16..256 (power of 2) and the 16-snap window, no
   * window, or a vec8 window with a non-increasing slice table and query-head
   * groups of at most 8. */
  int k_level_major;
  int64_t k_stride_page, k_stride_head, k_stride_level; /* elements; the token stride is 16 */
  /* Programmatic dependent launch (optional, 0 = off): the split kernel may
   * start while the previous kernel on the stream is still running. Before it
   * waits for that kernel it reads only items, item_indptr, indptr, indices and
   * last_page_len, so a kernel that writes one of those must not directly
   * precede the decode on the stream when this is set; q, q_pos, kv_pos0, the
   * KV pages and the outputs are read or written after the wait. */
  int enable_pdl;
} AtfDecodeParams;

/* Paged-KV GQA split-KV decode followed by the LSE merge of its splits. */
int atf_decode_run(const AtfDecodeParams* p, atf_stream_t stream);

/* atf_decode_run without any allocation. It has no counterpart in the
 * reference, whose decode always takes a workspace that the caller allocated.
 *
 * Who needs it: callers that cannot call cudaMalloc. Examples are a serving
 * engine that gave all free device memory to its KV-cache pool up front, and a
 * host whose step loop must not allocate because cudaMalloc and cudaFree
 * synchronise the device. Here the split workspace (partial_o, partial_lse)
 * comes from one fixed scratch array compiled into this library, one per
 * device. The function itself calls no cudaMalloc, cudaFree or allocating
 * library routine.
 *
 * Rules:
 *  - p->partial_o and p->partial_lse must be NULL. Every other field means what
 *    it means for atf_decode_run.
 *  - Limit: num_items * num_qo_heads <= ATF_NOALLOC_MAX_PARTIAL_ROWS. Larger
 *    plans return ATF_ERR_WORKSPACE and launch nothing; plan them with a larger
 *    min_chunk_keys, or use atf_decode_run.
 *  - Nothing in the scratch has to start at zero: each call writes every row it
 *    reads. The caller's error_flag, when given, must be zero on entry, as for
 *    atf_decode_run.
 *  - All calls on one device share the scratch. Calls that overlap on the GPU
 *    (on different streams with no ordering between them, or from several
 *    threads) race and corrupt each other's output. Issue them on one stream,
 *    or order them with events.
 *  - The first call in each CUDA context looks up the scratch address with
 *    cudaGetSymbolAddress (a context is told apart by its cuCtxGetId, so a
 *    device reset or a caller-made context gets its own lookup). Make that
 *    first call before any stream capture begins in that context.
 *  - item_indptr[batch_size] must equal num_items, as atf_decode_plan writes
 *    it; the merge never reads a part at or past num_items. */
#define ATF_NOALLOC_MAX_PARTIAL_ROWS 16384 /* 8 MiB + 64 KiB of fp32 scratch per device */
int atf_decode_run_noalloc(const AtfDecodeParams* p, atf_stream_t stream);

/* ------------------------------------------------------------------ merge */

typedef struct {
  const float* part_o;   /* ragged: [items, H, 128]; uniform: [P, B, H, 128] */
  const float* part_lse; /* ragged: [items, H]; uniform: [P, B, H] */
  const int32_t* part_indptr; /* device [B+1] for ragged parts; NULL for uniform P parts */
  int32_t num_parts;     /* uniform case: P */
  int32_t batch, num_heads, head_dim;
  int lse_log2;          /* 1: part_lse in log2 domain, 0: natural log */
  void* out;             /* [B, H, 128] */
  int64_t o_stride_b, o_stride_h;
  int out_dtype;         /* ATF_DTYPE_* */
  float* lse_out;        /* optional [B, H], natural log */
  /* Uniform parts only: floats between consecutive parts of part_o / part_lse
   * (0 = packed). A part's own [B, H, 128] / [B, H] block stays contiguous, so
   * parts gathered into one flat buffer per rank merge in place. part_stride_o
   * must be a multiple of 4. */
  int64_t part_stride_o, part_stride_lse;
} AtfMergeParams;

/* Merge partial attention states: LSE = log sum exp(LSE_i), O = sum exp(LSE_i - LSE) O_i. */
int atf_lse_merge(const AtfMergeParams* p, atf_stream_t stream);

/* ------------------------------------------------------------------ cross-rank state exchange */

/* No counterpart in the reference, which runs on one GPU. The KV-sharded decode
 * (the KV sequence split over the GPUs of one node) ends with every rank
 * holding a partial state (O fp32 [B, H, 128], LSE natural log [B, H]); these
 * calls merge the states of all ranks without a collective library: each rank
 * pushes its state into every peer's exchange region with NVLink peer stores
 * (no multicast), then merges once every peer's push of the step has arrived.
 * The merge is the same arithmetic as atf_lse_merge on uniform parts, so the
 * result is bit-identical to all-gathering the states and merging them.
 *
 * Exchange region: atf_exchange_region_bytes(B, H, world) bytes of device
 * memory per rank, 256-byte aligned, zeroed once before the first step, and
 * mapped into every other rank's process (atf_ipc_export / atf_ipc_import).
 * Every rank calls atf_state_push and then atf_state_merge once per step, in
 * the same order on one stream; the step counter lives in the region. A peer
 * that does not push within the wait limit (2 s) leaves ATF_ERR_TIMEOUT's code
 * in *error_flag and the merge returns without waiting further. */
#define ATF_IPC_HANDLE_BYTES 64
typedef struct {
  const float* o;       /* this rank's state: fp32 [B, H, 128] (16-byte aligned) */
  const float* lse;     /* fp32 [B, H], natural log, contiguous */
  int64_t o_stride_b, o_stride_h;
  int32_t batch, num_heads, world, rank;
  void* const* peer_base; /* device array [world]: every rank's region as mapped here (own at [rank]) */
  void* base;             /* this rank's region */
  void* out;              /* [B, H, 128], bf16 or fp32 */
  int64_t out_stride_b, out_stride_h;
  int out_dtype;
  float* lse_out;         /* optional [B, H], natural log */
  int* error_flag;        /* optional device int */
} AtfExchangeParams;

int64_t atf_exchange_region_bytes(int32_t batch, int32_t num_heads, int32_t world);
/* Push this rank's state into slot [step parity][rank] of every rank's region and
 * signal each of them. */
int atf_state_push(const AtfExchangeParams* p, atf_stream_t stream);
/* Wait (bounded) for every rank's push of this step, merge, advance the step. */
int atf_state_merge(const AtfExchangeParams* p, atf_stream_t stream);
/* One KV-sharded decode step with the exchange fused into the decode's own
 * split merge: atf_decode_run(p) whose merge kernel also stores this rank's
 * state into every rank's region (as atf_state_push), waits (bounded) for
 * every peer's state of the step and writes the merge of all ranks' states to
 * p->out / p->lse_out (as atf_state_merge). One kernel follows the decode
 * instead of three; the outputs are bit-identical to atf_decode_run with fp32
 * out and lse, atf_state_push and atf_state_merge. Uses x's batch, num_heads,
 * world, rank, peer_base, base and error_flag (p->error_flag when NULL); x's
 * o, lse and out fields are not read. Every rank of the exchange calls it once
 * per step; the ranks of one exchange must run on different GPUs, since each
 * rank's kernel waits for the others'. */
int atf_decode_run_exchange(const AtfDecodeParams* p, const AtfExchangeParams* x, atf_stream_t stream);
/* CUDA IPC of a device allocation: the handle of the allocation holding dev_ptr
 * and dev_ptr's offset in it; import maps a peer's handle (ptr = base + offset);
 * release unmaps a base returned by import. Setup calls, not for the step loop. */
int atf_ipc_export(const void* dev_ptr, void* handle_out, int64_t* offset_out);
int atf_ipc_import(const void* handle, int64_t offset, void** ptr_out, void** base_out);
int atf_ipc_release(void* base);

/* ------------------------------------------------------------------ RoPE */

typedef struct {
  const void* x; /* bf16 [B, S, H, 128], pre-RoPE, rotate_half pair order */
  void* out;     /* bf16 [B, S, H, 128] */
  int64_t batch, seqlen, num_heads, head_dim;
  int64_t x_stride_b, x_stride_s, x_stride_h;
  int64_t o_stride_b, o_stride_s, o_stride_h;
  const float* cos; /* fp32 [n_pos, 64]: row p = cos(p * inv_freq) */
  const float* sin;
  int64_t cs_stride_pos; /* elements between consecutive positions */
  int64_t n_pos;
  const int64_t* positions; /* optional device [S]; default pos_offset + s */
  int64_t pos_offset;
  int out_layout; /* ATF_LAYOUT_SORTED_PAIR or ATF_LAYOUT_ROTATE_HALF */
} AtfRopeParams;

/* rotate_half RoPE in fp32 (x1*cos - x2*sin, x2*cos + x1*sin, no FMA
 * contraction), rounded to bf16, written in the requested pair order. */
int atf_rope_pack(const AtfRopeParams* p, atf_stream_t stream);

/* ------------------------------------------------------------------ paged-KV append */

typedef struct {
  const void* append_k; /* bf16 [nnz, Hkv, 128]: pre-RoPE HF rotate_half order when cos/sin are given */
  const void* append_v; /* bf16 [nnz, Hkv, 128] */
  int64_t nnz;
  int64_t a_stride_n, a_stride_h; /* same for append_k and append_v */
  const int32_t* batch_indices;   /* device [nnz]: request of each token */
  const int32_t* positions;       /* device [nnz]: position of the token in its request's KV */
  void* k_cache;                  /* bf16 pages, NHD [P, page, Hkv, 128] or HND [P, Hkv, page, 128] */
  void* v_cache;
  int64_t num_pages;
  int64_t kv_stride_page, kv_stride_token, kv_stride_head;
  int32_t num_kv_heads, head_dim, page_size, batch_size;
  const int32_t* kv_indptr;       /* device [B+1] */
  const int32_t* kv_indices;      /* device page ids */
  const float* cos;               /* optional fp32 [n_pos, >=64]: rotate K at write */
  const float* sin;
  int64_t cs_stride_pos, n_pos;
  const int64_t* rope_positions;  /* optional device [nnz]: RoPE position (default: positions[i]) */
  int out_layout;                 /* with RoPE: pair order written (ATF_LAYOUT_*) */
  int* error_flag;                /* optional: set to 2 when a token's page index is out of range */
  /* Level-major K pages (see AtfDecodeParams): K is written as [P, Hkv, 8, page, 16]
   * in sorted-pair order (with RoPE, out_layout must be sorted pair). */
  int k_level_major;
  int64_t k_stride_page, k_stride_head, k_stride_level;
} AtfAppendParams;

/* Append K/V tokens to a paged cache: token i goes to page
 * kv_indices[kv_indptr[b] + pos / page], slot pos % page (b = batch_indices[i],
 * pos = positions[i]); with cos/sin, K is rotated and packed into out_layout.
 * Replaces FlashInfer's append_paged_kv_cache, which feeds the reference's
 * decode (e2e_pipeline/atflash_e2e_fafi.py:219-223). */
int atf_paged_kv_append(const AtfAppendParams* p, atf_stream_t stream);

/* ------------------------------------------------------------------ misc */

const char* atf_status_string(int status);
int atf_version(void);
/* sizeof of the named params struct ("AtfPrefillParams", "AtfDecodePlanParams",
 * "AtfDecodePlan", "AtfDecodeParams", "AtfMergeParams", "AtfRopeParams",
 * "AtfAppendParams", "AtfExchangeParams"), or -1: lets an FFI binding check its struct mirrors. */
int64_t atf_params_size(const char* name);
/* Synchronises the current device, copies *error_flag to *out and clears it. */
int atf_read_error_flag(int* error_flag_device, int* out);

/* Self-test of the bounded device waits (no counterpart in the reference, which
 * has no device-side waits): launches one thread that waits on an mbarrier that
 * nothing arrives on. After the wait limit (2 s) the kernel writes 1 to
 * *error_flag and returns; the context stays usable. Failure detection is
 * tested this way instead of with a fault. */
int atf_selftest_wait_timeout(int* error_flag_device, atf_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* ATFLASH_B200_H_ */
