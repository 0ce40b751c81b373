/*
 * flashdec_b200 -- C ABI of the B200 (sm_100a) paged-decode data path.
 *
 * This is the drop-in boundary: plain pointers, element strides and sizes,
 * no framework types.  Every entry point returns 0 (FD_OK) or a negative
 * FD_ERR_* code; nothing allocates device memory, nothing synchronises the
 * stream, and all work is enqueued on the caller's stream.
 *
 * Reference interfaces replaced (paths inside cysong2025/flashdec):
 *
 *   fd_paged_decode      <- the Triton launches of
 *                           flashdec/kernels/paged_decode.py:922-1264
 *                           (paged_decode_attention / _into: the grouped-GQA
 *                           kernel :124-327, the split kernel :330-543 and the
 *                           per-head MHA kernel :28-121) and the unchecked
 *                           vLLM launcher :728-919 (fused current-token append,
 *                           slot_mapping == -1 padding rows).
 *   fd_split_kv_reduce   <- _paged_decode_gqa_reduce_kernel,
 *                           flashdec/kernels/paged_decode.py:546-642.
 *   fd_rope_kv_append    <- pybind fused_rope_kv_append,
 *                           flashdec/csrc/fused_rope_kv_append.cpp:90-132
 *                           (kernel .cu:38-139), and pybind kv_append,
 *                           flashdec/csrc/kv_append.cpp:60-73 (kernel
 *                           kv_append_kernel.cu:10-84) when q == NULL and
 *                           rotary_dim == 0.
 *
 * Threading: entry points are re-entrant; per-device state (SM count, tensor
 * map cache) is initialised once under a lock.  Calls that share a workspace
 * must be ordered on one stream.
 */
#ifndef FLASHDEC_B200_H_
#define FLASHDEC_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define FD_OK 0
#define FD_ERR_INVALID_ARGUMENT (-1)  /* null pointer, bad rank/size      */
#define FD_ERR_UNSUPPORTED (-2)       /* dtype / head_dim / block_size     */
#define FD_ERR_WORKSPACE (-3)         /* workspace missing or too small    */
#define FD_ERR_CUDA (-4)              /* a CUDA runtime call failed        */
#define FD_ERR_ALIGNMENT (-5)         /* pointer/stride alignment          */
#define FD_ERR_CAPACITY (-6)          /* need exceeds fd_paged_decode_static's
                                         static storage                    */

/* device status word bits (fd_device_status) */
#define FD_STATUS_WAIT_TIMEOUT 1      /* a bounded mbarrier wait ran out   */
#define FD_STATUS_BAD_BLOCK_ID 2      /* a block id outside [0, num_blocks)
                                         was met inside seq_len and masked */

/* ---- dtypes ------------------------------------------------------------ */
#define FD_DTYPE_F32 0
#define FD_DTYPE_F16 1
#define FD_DTYPE_BF16 2
#define FD_INDEX_I32 0
#define FD_INDEX_I64 1

/* ---- paged decode attention -------------------------------------------- */
#define FD_EPILOGUE_FUSED 0      /* split partials merged inside the kernel */
#define FD_EPILOGUE_PARTIALS 1   /* write partials only; fd_split_kv_reduce */

typedef struct fd_paged_decode_args {
  int32_t struct_size;   /* = sizeof(fd_paged_decode_args) */
  int32_t dtype;         /* FD_DTYPE_F16 or FD_DTYPE_BF16 (q, caches, out) */
  int32_t num_seqs;      /* rows of q launched (vLLM num_reqs incl. padding) */
  int32_t num_q_heads;
  int32_t num_kv_heads;  /* num_q_heads % num_kv_heads == 0 */
  int32_t head_dim;      /* 64 or 128 */
  int32_t block_size;    /* 8, 16 or 32 tokens per page */
  int32_t num_blocks;    /* physical pages in the cache */
  int32_t max_blocks_per_seq; /* block-table row length */
  float sm_scale;

  /* q [num_seqs, num_q_heads, head_dim], out the same (element strides) */
  const void* q;
  int64_t q_stride[3];
  void* out;
  int64_t out_stride[3];

  /* caches, logical order [block, kv_head, token, dim] (element strides);
   * token-major, dim-major, vLLM NHD/HND planes are all expressible. */
  void* k_cache;
  int64_t k_stride[4];
  void* v_cache;
  int64_t v_stride[4];

  const void* block_tables;      /* [num_seqs, max_blocks_per_seq] */
  int32_t block_tables_index;    /* FD_INDEX_I32 / FD_INDEX_I64 */
  int64_t block_tables_stride[2];
  const void* seq_lens;          /* [num_seqs] */
  int32_t seq_lens_index;
  int64_t seq_lens_stride;

  /* optional fused append of the current token (append_k == NULL: off).
   * Token seq_len-1 of row s comes from append_k/v[s] and is stored at
   * slot_mapping[s] = block * block_size + offset; rows with slot < 0 get a
   * zero output and no store. */
  const void* append_k;
  int64_t append_k_stride[3];
  const void* append_v;
  int64_t append_v_stride[3];
  const void* slot_mapping;
  int32_t slot_mapping_index;
  int64_t slot_mapping_stride;

  /* work decomposition */
  int32_t num_splits;    /* 0: auto (length-balanced over the whole batch);
                            S >= 1: S splits of every sequence (reference) */
  int32_t epilogue;      /* FD_EPILOGUE_FUSED / FD_EPILOGUE_PARTIALS */
  /* partial layout for num_splits >= 1: acc [seq, q_head, split, dim],
   * max/sum [seq, q_head, split] (fp32, element strides, max in natural-log
   * units of the scaled scores).  NULL: use the internal workspace. */
  float* part_acc;
  int64_t part_acc_stride[4];
  float* part_max;
  float* part_sum;
  int64_t part_stat_stride[3];

  /* Caller-owned scratch, reused across calls (see fd_paged_decode_workspace):
   *   tickets  int32 [tickets_capacity], zero-filled ONCE by the caller; the
   *            kernel leaves every entry at zero when it returns;
   *   scratch  fp32 partials, no initialisation needed. */
  int32_t* tickets;
  int64_t tickets_capacity;
  float* scratch;
  size_t scratch_bytes;
  int32_t max_ctas;          /* 0: one CTA per SM */
  int32_t min_tiles_per_cta; /* 0: default (4); auto schedule only */

  /* optional split-half RoPE of the fused-append row (needs append_k; 0: off).
   * q[s] and append_k[s] are rotated by position rope_positions[s] with the
   * fp32 table rope_inv_freq[rope_dim / 2] (= base^(-2i/rope_dim), computed
   * like flashdec/rope.py:66-67), exactly as fd_rope_kv_append rotates them;
   * the rotated K row is what the cache slot receives.  One launch then does
   * a whole decode layer of flashdec/engine.py:1072-1183 (RoPE + K/V store
   * + paged attention). */
  int32_t rope_dim;
  const float* rope_inv_freq;
  const void* rope_positions;
  int32_t rope_positions_index;
  int64_t rope_positions_stride;
} fd_paged_decode_args;

/* Workspace needed by fd_paged_decode for `args`: scratch bytes and ticket
 * entries (both 0 when the call needs none). */
int fd_paged_decode_workspace(const fd_paged_decode_args* args, size_t* scratch_bytes,
                              int64_t* tickets_needed);

int fd_paged_decode(const fd_paged_decode_args* args, void* cuda_stream);

/* ---- cascade (shared-prefix) decode -----------------------------------------
 * Same result as fd_paged_decode(args) for a batch in which groups of
 * sequences share the first pages of their block-table rows (a prompt prefix
 * registered once and attached to every member: flashdec/cache.py:192-276).
 * The shared pages are read once per KV head for all of a group's query rows
 * (prefix pass, 128 rows per CTA, one partial per chunk of pages); the rest of
 * every sequence goes through the split decode (tail pass).  By default the
 * prefix pass runs on a second stream of the library's own beside the tail
 * pass on the caller's stream (fork and join by events: capturable), and one
 * reduction then merges each row's tail and prefix partials (LSE merge of
 * flashdec/kernels/paged_decode.py:593-635): three launches.  The second
 * stream and its two events are created by the first such call on a device
 * (that device current; make it before any stream capture); calls from
 * several host threads take turns on them.  With
 * FLASHDEC_B200_CASCADE_CONCURRENT=0 the two passes run one after the other
 * on the caller's stream and the tail's last CTA per (sequence, head block)
 * merges through the tickets: two launches.  args->num_splits, epilogue and part_* are
 * ignored; args->scratch and args->tickets must hold fd_cascade_workspace's
 * sizes (tickets zero-filled once; the kernels leave them zero).  The group
 * description lives in HOST memory and is copied into the launch; every
 * member's seq_len must exceed its group's prefix tokens (its current token
 * is private).  FD_ERR_UNSUPPORTED for caches the TMA loader cannot address
 * or more than 32 groups / 512 members (call fd_paged_decode instead). */
typedef struct fd_cascade_args {
  int32_t struct_size;             /* = sizeof(fd_cascade_args) */
  int32_t num_groups;              /* 1..32 */
  const int32_t* group_start;      /* host [num_groups + 1]: CSR offsets into group_members */
  const int32_t* group_members;    /* host: sequence indices (rows of q), grouped, <= 512 */
  const int32_t* group_pages;      /* host [num_groups]: shared pages, pages * block_size % 32 == 0 */
  const int32_t* seq_prefix_pages; /* DEVICE [num_seqs]: the sequence's group_pages, 0 outside */
  int32_t chunks;                  /* prefix chunks per (group, kv head, 128 rows); 0: auto */
  int32_t tail_splits;             /* splits of every sequence's tail; 0: auto */
} fd_cascade_args;

int fd_cascade_workspace(const fd_paged_decode_args* args, const fd_cascade_args* cascade,
                         size_t* scratch_bytes, int64_t* tickets_needed);
int fd_cascade_decode(const fd_paged_decode_args* args, const fd_cascade_args* cascade,
                      void* cuda_stream);

/* fd_paged_decode with its ticket and scratch buffers taken from 8 MiB of
 * fp32 scratch and 4096 int32 tickets that are static device storage of the
 * library (the tickets/scratch fields of `args` are ignored), for callers
 * that cannot allocate device memory.  No counterpart in the reference.
 * - The first call on a device (that device current) looks up the storage
 *   address, and so does the first call after the device's context changed
 *   (cudaDeviceReset); make those calls before any stream capture.
 * - FD_EPILOGUE_PARTIALS needs the caller's part_acc / part_max / part_sum
 *   (the static scratch is private): a NULL part_acc returns
 *   FD_ERR_INVALID_ARGUMENT.
 * - The tickets start at zero (zero-filled at module load) and every
 *   completed call leaves them at zero; after a call that raised
 *   FD_STATUS_WAIT_TIMEOUT, do not use this entry point again.
 * - All calls on a device share the storage: calls that overlap on the GPU
 *   race; order them (e.g. one stream).
 * - A call needing more than the static storage (see
 *   fd_paged_decode_workspace) returns FD_ERR_CAPACITY and launches nothing. */
int fd_paged_decode_static(const fd_paged_decode_args* args, void* cuda_stream);

/* Diagnostic: launch one warp that waits, through the kernels' bounded
 * mbarrier wait, on a barrier nothing arrives on, for `limit_ns` (1 ns .. 5 s).
 * It then raises FD_STATUS_WAIT_TIMEOUT in the device status word and returns;
 * the context stays usable.  Used to test the failure path without a GPU
 * fault.  No counterpart in the reference. */
int fd_selftest_wait_timeout(int64_t limit_ns, void* cuda_stream);

/* ---- split-KV reducer --------------------------------------------------- */
typedef struct fd_split_kv_reduce_args {
  int32_t struct_size;
  int32_t dtype;         /* of out */
  int32_t num_seqs;
  int32_t num_q_heads;
  int32_t head_dim;
  int32_t num_splits;
  const float* part_acc;
  int64_t part_acc_stride[4];
  const float* part_max;
  const float* part_sum;
  int64_t part_stat_stride[3];
  const void* seq_lens;
  int32_t seq_lens_index;
  int64_t seq_lens_stride;
  const void* slot_mapping;  /* optional: slot < 0 rows are zeroed */
  int32_t slot_mapping_index;
  int64_t slot_mapping_stride;
  void* out;
  int64_t out_stride[3];
} fd_split_kv_reduce_args;

int fd_split_kv_reduce(const fd_split_kv_reduce_args* args, void* cuda_stream);

/* ---- fused RoPE + paged K/V append --------------------------------------
 * With num_kv_heads == 0 (and q given) the call only rotates q into q_out:
 * k, v, the caches and the index pointers may then be NULL and positions is
 * the only index read.  This is the native form of flashdec/rope.py:26-85
 * (apply_rope) for device tensors. */
typedef struct fd_rope_kv_append_args {
  int32_t struct_size;
  int32_t dtype;          /* FD_DTYPE_F32 / F16 / BF16 */
  int32_t batch;          /* tokens (one per request) */
  int32_t num_q_heads;    /* 0 when q == NULL */
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t rotary_dim;     /* even, <= head_dim; 0 = copy K unrotated */
  int32_t block_size;
  int32_t num_blocks;
  const float* inv_freq;  /* [rotary_dim/2] fp32 device table (rotary_dim>0) */
  const void* q;          /* optional [batch, num_q_heads, head_dim] */
  int64_t q_stride[3];
  void* q_out;
  int64_t q_out_stride[3];
  const void* k;          /* [batch, num_kv_heads, head_dim] */
  int64_t k_stride[3];
  const void* v;
  int64_t v_stride[3];
  void* k_cache;          /* [block, kv_head, token, dim] */
  int64_t k_cache_stride[4];
  void* v_cache;
  int64_t v_cache_stride[4];
  const void* block_ids;  /* [batch] */
  const void* block_offsets;
  const void* positions;  /* [batch]; required when q != NULL or rotary_dim > 0 */
  int32_t block_ids_index;
  int32_t block_offsets_index;
  int32_t positions_index;
  int32_t reserved;
} fd_rope_kv_append_args;

int fd_rope_kv_append(const fd_rope_kv_append_args* args, void* cuda_stream);

/* ---- misc ---------------------------------------------------------------- */
const char* fd_error_string(int code);
int fd_version(void);
/* Synchronous read (and optional clear) of the current device's status word. */
int fd_device_status(int clear, int* status_out);
/* Number of SMs of the current device (cached). */
int fd_num_sms(void);

#ifdef __cplusplus
}
#endif

#endif /* FLASHDEC_B200_H_ */
