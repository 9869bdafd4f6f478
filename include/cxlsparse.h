/*
 * cxlsparse_b200 C ABI: the drop-in boundary for the NSA generative-
 * recommendation selected-block path of Sispheqgj/cxlsparse, rebuilt for
 * B200 (sm_100a).
 *
 * Conventions
 *  - Plain pointers and sizes only; every device pointer is a CUDA device (or
 *    UVA host-mapped) address on the current device; `stream` is a
 *    cudaStream_t passed as void*.
 *  - Every entry point returns CXS_OK (0) or a CXS_ERR_* code and never
 *    throws. cxs_last_error() returns a thread-local message for the last
 *    failure on the calling thread.
 *  - Launch entry points only enqueue work on `stream`: no host
 *    synchronisation, no device allocation, no host<->device copies, so they
 *    can be captured in a CUDA graph (the reference captures plan + execute,
 *    models/nsa/transport.py:624-631).
 *  - Device-side failures (invalid selections, bounded-wait timeouts) are
 *    reported through device words the caller reads after the stream
 *    completes (planner stats column 6, and the `error` word of
 *    cxs_fetch_attend), mirroring DeferredLayerCounters
 *    (mempool/device_plan.py:16-42).
 *
 * Reference citations are file:line within the reference project.
 */
#ifndef CXLSPARSE_B200_H
#define CXLSPARSE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CXS_ABI_VERSION 4

enum cxs_status {
  CXS_OK = 0,
  CXS_ERR_INVALID = 1,      /* bad geometry / argument (reference: ValueError) */
  CXS_ERR_CUDA = 2,         /* a CUDA runtime call failed */
  CXS_ERR_CAPACITY = 3,     /* capacity refusal before any side effect
                               (reference: GRWorkspaceLimit, transport.py:24-25) */
  CXS_ERR_REGISTRATION = 4, /* host pool registration failed */
  CXS_ERR_UNSUPPORTED = 5   /* device lacks a required feature */
};

/* Bits of the device error word written by cxs_fetch_attend. */
#define CXS_DEVICE_ERR_READY_TIMEOUT 1 /* an attention engine gave up waiting on ready[b] */
#define CXS_DEVICE_ERR_COPY_TIMEOUT 2  /* a bulk copy did not complete within the limit */
#define CXS_DEVICE_ERR_BAD_BLOCK 4     /* a plan entry was out of range */

/* Read-order policies (planning/read_order.py:11-18). */
#define CXS_ORDER_PHYSICAL 0
#define CXS_ORDER_DEPTH 1        /* "consumption_depth" */
#define CXS_ORDER_DEPTH_SHARED 2 /* "consumption_depth_shared" */

int cxs_abi_version(void);
const char* cxs_last_error(void);
/* Kernels this library has enqueued so far in this process (diagnostic; a
 * CUDA-graph replay re-runs captured launches without counting them again). */
int64_t cxs_launch_count(void);

/* ------------------------------------------------------------------ pool ---
 * Backing pool outside HBM: NUMA-local pinned host memory, registered for
 * mapped device access with device VA == host VA.
 */

/* Allocate `bytes` of anonymous host memory bound to NUMA node `numa_node`
 * (-1: the node of CUDA device `device`, or no binding if unknown), touch it,
 * and register it with cudaHostRegister(Mapped|Portable).
 * Replaces the DRAM pool mapping + registration of mempool/pool.py:60 and
 * mempool/native/cuda_registration.cuh:19-40. */
int cxs_pool_create(size_t bytes, int device, int numa_node, void** host_base,
                    int* bound_node);
/* Unregister and unmap memory returned by cxs_pool_create. */
int cxs_pool_destroy(void* host_base, size_t bytes);
/* Register caller-owned host memory (mempool/native/cuda_registration.cuh:19-40):
 * fails unless the device pointer equals the host pointer. */
int cxs_pool_register(void* host_base, size_t bytes);
/* Undo cxs_pool_register (mempool/native/cuda_registration.cuh:43-47). */
int cxs_pool_unregister(void* host_base);
/* NUMA node of a CUDA device's PCI function, or -1 if unknown. */
int cxs_device_numa_node(int device);

/* Scatter `count` bf16 KV records [count, 128] from device memory into pool
 * token slots (page-striped over `regions` region bases). Replaces the region
 * write kernel (mempool/native/region_write.cuh:14-51, mempool/cxl.py:194-228). */
int cxs_pool_write(const void* records, const int64_t* slots, int64_t count,
                   const int64_t* region_bases, int regions, int page_size,
                   void* stream);

/* -------------------------------------------------------------- planner ---
 * Device-side fetch planner (planning/active.py:670-907 for the
 * deduplicating plan; planning/query_private.py:258-457 for the no-dedup
 * plan). Array meanings and layouts equal the reference workspace entries of
 * the same name (planning/active.py:554-611).
 */
typedef struct cxs_plan_geometry {
  int32_t queries;       /* token rows Q (row r = q * heads + head) */
  int32_t heads;         /* KV heads H */
  int32_t width;         /* selected blocks per row W */
  int32_t block_size;    /* BS, a power of two */
  int32_t map_blocks;    /* MAP: logical block capacity */
  int32_t per_head;      /* CAP: compact slots per head */
  int32_t sort_extent;   /* frequency table length per head */
  int32_t hot;           /* hot replica tokens per cache row */
  int32_t max_history;   /* host_locs row length */
  int32_t regions;       /* pool region count */
  int32_t page_size;     /* pool page size (tokens) */
  int32_t consumer_ctas; /* consumers assumed by the depth order */
  int32_t read_order;    /* CXS_ORDER_* */
  int32_t private_plan;  /* 0 = dedup across rows, 1 = query-private */
  int32_t launch_mode;   /* 0: a deduplicating plan runs as one launch of a
                            single thread-block cluster when its tables fit
                            (otherwise, and for 1, one launch per phase) */
  int64_t pool_tokens;   /* pool capacity in token slots */
} cxs_plan_geometry;

typedef struct cxs_plan_buffers {
  /* inputs */
  const int32_t* blocks;    /* [Q, H, W] selected block ids, -1 padded */
  const int32_t* positions; /* [Q] absolute positions, -1 = padded row */
  const int64_t* desc;      /* [H, 5] (cache row, cached_len, history_len,
                               current_kv address, current_len) */
  const int64_t* bases;     /* [regions] pool region base addresses */
  const int32_t* tags;      /* cache tags [rows, hot + 1] */
  const int32_t* locs;      /* cache locations [rows, hot + 1] */
  const int64_t* host_locs; /* cache token -> pool slot [rows, max_history] */
  const void* hot_data;     /* cache hot KV data [rows * (hot + 1), 128] bf16 */
  /* persistent + scratch (device) */
  int32_t* mapping;         /* dedup: [H, MAP + 1]; private: [H, CAP] */
  int32_t* insert_keys;     /* [H, CAP] */
  int32_t* active_keys;     /* [H, CAP] */
  int32_t* active_counts;   /* [H] */
  int32_t* required;        /* [H, CAP] */
  int32_t* frequencies;     /* [H, sort_extent] */
  int32_t* stats;           /* [H, 7] */
  int64_t* address;         /* [P, BS] */
  int64_t* hbm;             /* [P, BS] */
  int32_t* valid;           /* [P] */
  int32_t* starts;          /* [P] */
  int32_t* flags;           /* [P] missing */
  int64_t* slots;           /* [P * BS] */
  int32_t* ioids;           /* [P] */
  int32_t* ranks;           /* [P] */
  int32_t* missing;         /* [1] */
  int32_t* all_ids;         /* [R, W] */
  int32_t* all_counts;      /* [R] */
  int32_t* row_positions;   /* [R] */
  int32_t* region_counts;   /* [regions] */
  int32_t* row_depth;       /* [R] */
  int32_t* first_depth;     /* [P] first consumption depth of every referenced block */
  int32_t* near_consumers;  /* [P] near consumers of every referenced block */
  int32_t* chosen;          /* [H, hot] chosen hot indices */
  /* query-private plan only (may be NULL otherwise) */
  int32_t* private_required;    /* [H, CAP] */
  int32_t* private_occurrences; /* [R, W] */
  int32_t* canonical;           /* [H, sort_extent] */
  /* optional HBM residency table (NULL: the hot tags/locs hash). When set,
   * history token t of cache row r is resident at hot_data +
   * hbm_locs[r * max_history + t] * 256 if that entry is >= 0, else it comes
   * from the backing pool; tags/locs are not read. Any residency pattern
   * (a recency window of any size, interleaved or partial blocks) is a
   * table. No counterpart in the reference, whose replica is the hot hash. */
  const int32_t* hbm_locs;      /* [rows, max_history] */
} cxs_plan_buffers;


/* Bytes of dynamic shared memory / limits check for a geometry; returns
 * CXS_ERR_CAPACITY for geometries the kernels refuse (before any launch). */
int cxs_plan_check(const cxs_plan_geometry* geometry);

/* Enqueue the whole plan: reset, dedup insert, sorted compaction, references,
 * per-token source resolution, missing-block ranks, occurrence rows,
 * read order, and the hot top-k choice. */
int cxs_plan(const cxs_plan_geometry* geometry, const cxs_plan_buffers* buffers,
             void* stream);

/* cxs_plan without the hot top-k choice, for callers that run the choice
 * and the commit later (for example on a second stream, overlapped with the
 * next layer) through cxs_plan_select_commit_hot. */
int cxs_plan_core(const cxs_plan_geometry* geometry, const cxs_plan_buffers* buffers,
                  void* stream);

/* Hot top-k choice followed by cxs_plan_commit_hot (pairs with cxs_plan_core). */
int cxs_plan_select_commit_hot(const cxs_plan_geometry* geometry,
                               const cxs_plan_buffers* buffers, const void* kv, int32_t* tags,
                               void* hot_data, void* stream);

/* Commit the chosen hot tokens once attention has completed: write tags and
 * copy their KV from the staging buffer `kv` [P, BS, 128] bf16 into the
 * cache hot data (planning/active.py:410-437, 909-925;
 * planning/query_private.py:188-216). */
int cxs_plan_commit_hot(const cxs_plan_geometry* geometry, const cxs_plan_buffers* buffers,
                        const void* kv, int32_t* tags, void* hot_data, void* stream);

/* ------------------------------------------------ IO + attention kernel ---
 * One persistent launch with two warp roles (tma/transport.py:17-112 and
 * tma/pipeline.py:96-742 are the reference's prepare + staged TMA kernel):
 *  - IO warps take missing blocks in IOIDs order from a device cursor; full
 *    contiguous 16-byte aligned external blocks move host -> shared -> HBM
 *    with 1-D bulk TMA copies, mixed/tail blocks move with 16-byte vector
 *    gathers; each then publishes ready[b] with st.release.gpu.
 *  - attention engines (warp pairs) own query rows; they first run the
 *    sliding-window branch (HBM resident), then acquire ready[b] for each
 *    selected occurrence in the original order (not needed for blocks that
 *    were resident before the launch), stage K and V through shared memory
 *    with 2-D tensor TMA, and run online-softmax attention with tcgen05 MMAs
 *    that the engine warp issues while its softmax warp works on the
 *    previous tile; the epilogue optionally applies the sigmoid-gate mix
 *    (models/nsa/model.py:470-473).
 * A preceding prepare kernel (same call) classifies block sources, gathers
 * resident blocks into the staging buffer and initialises ready flags.
 */
/* Candidate segments. The reference packs every GR candidate into one suffix
 * (worker/prompt.py:24-55), so candidates attend to each other's tokens.
 * With segment_tokens > 0 several candidates instead share one history and
 * each sees only the history and its own suffix:
 *  - positions below segment_start (a multiple of the block size) are
 *    history, shared by all candidates;
 *  - candidate s's suffix token with true position segment_start + i sits at
 *    position segment_start + s * segment_tokens + i (segment_tokens is a
 *    multiple of the block size, at least the candidate's suffix length);
 *  - a row whose position p lies in segment s > 0 sees history positions
 *    below segment_start and its own segment up to p; segments 1..s-1 and
 *    the start of segment 0 beyond the history are a gap it never reads.
 * Blocks, summaries, window records and current KV use these positions,
 * so the planner deduplicates history blocks across candidates and keeps
 * each candidate's suffix blocks private without knowing about segments.
 * The window branch covers the true positions (p_true - window, p_true]. */
typedef struct cxs_attend_geometry {
  int32_t queries;      /* Q token rows */
  int32_t heads;        /* H */
  int32_t width;        /* W */
  int32_t block_size;   /* BS in {16, 32, 64} */
  int32_t physical;     /* P = H * CAP */
  int32_t window;       /* sliding window W_s (0: no window branch) */
  int32_t window_len;   /* records in the window buffer */
  int32_t gate;         /* 1: write the gate mix instead of the selected output */
  int64_t window_start; /* absolute position of window record 0 (may be negative:
                           records before position 0 are never in a window) */
  int64_t spin_limit;   /* clock cycles before a bounded wait gives up */
  int64_t segment_start;  /* candidate segments (0, 0: one suffix): see below */
  int64_t segment_tokens;
  int32_t out_heads;  /* 0: `out` is [Q, H, 16, 64]; else [Q, out_heads, 16, 64] and this */
  int32_t out_head0;  /* call's heads are out_head0 .. out_head0 + H - 1 (KV-head split) */
  int32_t ctas;       /* 0: the IO/attention launch fills every SM; else at most this many
                         CTAs, leaving the other SMs to work on concurrent streams (the
                         fetch needs few CTAs to keep the host link busy). Any value is
                         correct; for the best read order the planner's consumer count
                         is min(rows, 4 * launched CTAs), cxs_attend_capacity giving
                         4 * the CTAs of an uncapped launch. */
} cxs_attend_geometry;

typedef struct cxs_attend_buffers {
  const void* query;         /* [Q, H, 16, 64] bf16 */
  void* kv;                  /* staging [P, BS, 128] bf16 */
  const int32_t* all_ids;    /* [R, W] */
  const int32_t* all_counts; /* [R] */
  const int32_t* row_positions; /* [R] */
  const int32_t* starts;     /* [P] */
  const int32_t* valid;      /* [P] */
  const int32_t* flags;      /* [P] missing */
  const int32_t* ioids;      /* [P] */
  const int32_t* missing;    /* [1] */
  const int64_t* address;    /* [P, BS] per-token source addresses */
  int64_t* sources;          /* [P] bulk source (or staging) per block */
  int32_t* kinds;            /* [P] 0 resident, 1 bulk, 2 gather */
  int32_t* ready;            /* [P] */
  int32_t* control;          /* [4] device cursor/scratch, reset by the call */
  int32_t* error;            /* [1] device error word (CXS_DEVICE_ERR_*), reset by the call */
  const void* window_kv;     /* [window_len, H, 128] bf16 or NULL */
  const void* compressed;    /* [Q, H, 16, 64] bf16 compressed-branch output (gate) */
  const void* gates;         /* [Q, H, 16, 3] bf16 sigmoid gates (gate) */
  void* out;                 /* [Q, H, 16, 64] bf16 (or out_heads, see the geometry) */
  void* out_peer;            /* NULL, or a peer GPU's buffer of the same layout: every
                                output row is also stored there over NVLink (KV-head
                                split exchange; see cxs_exchange_barrier) */
  const int32_t* first_depth;    /* [P] the plan's first consumption depth of every
                                    block (cxs_plan_buffers.first_depth), or NULL */
  const int32_t* near_consumers; /* [P] the plan's near-consumer counts, or NULL.
                                    With first_depth, every row takes its selected
                                    blocks by the read-order key (first depth, more
                                    near consumers first, block; ties in list order),
                                    the key the IO warps fetch missing blocks by, so
                                    an engine follows the order in which blocks
                                    arrive. The plan keys every block whatever its
                                    residency, so the result does not depend on
                                    residency; it differs from list order (NULL) by
                                    fp32 summation rounding. */
} cxs_attend_buffers;

int cxs_fetch_attend(const cxs_attend_geometry* geometry, const cxs_attend_buffers* buffers,
                     void* stream);

/* Number of attention engines (consumers) one cxs_fetch_attend launch runs on
 * the current device for `block_size` (grid = resident CTAs x 4 warp-pair
 * engines). A plan's consumer_ctas should be min(rows, this) so that its
 * consumption-depth order models the real consumers (tma/transport.py:63
 * uses min(rows, 256)). */
int cxs_attend_capacity(int32_t block_size, int32_t* attention_warps);

/* Allocation-free variant of cxs_fetch_attend. No counterpart in the
 * reference: it exists for callers that cannot allocate device memory
 * themselves, for example a plugin inside a host process whose own allocator
 * owns all of the GPU's memory, or code that must not call cudaMalloc after
 * start-up because cudaMalloc can synchronise the whole device.
 *
 * The caller passes the same geometry and buffers as for cxs_fetch_attend
 * (inputs, the staging buffer `kv`, `out` and the `error` word), but
 * `sources`, `kinds`, `ready` and `control` are ignored: that scratch lives in
 * a static device array of this library sized for CXS_NOALLOC_MAX_PHYSICAL
 * blocks (about 256 KiB on every GPU that loads the library, held until the
 * process exits). Larger geometries are rejected with CXS_ERR_CAPACITY.
 * The first call on each device looks up the array's device address with
 * that device current; make that first call before any stream capture.
 * All calls share the one array and each call re-initialises it, so calls
 * that overlap on the GPU (different streams, or another thread) race and
 * must be serialised by the caller. Nothing is allocated by this entry point. */
#define CXS_NOALLOC_MAX_PHYSICAL 16384
int cxs_fetch_attend_noalloc(const cxs_attend_geometry* geometry,
                             const cxs_attend_buffers* buffers, void* stream);

/* ------------------------------------------------ KV-head split exchange ---
 * The reference is single-GPU. When the two KV heads of a user are split over
 * a GPU pair, each attention launch stores its output rows into its own and
 * its peer's gather buffer (cxs_attend_buffers.out_peer, NVLink stores), and
 * cxs_exchange_barrier then tells the peer that its rows have landed and waits
 * (bounded) for the peer's. Buffers are shared with CUDA IPC.
 */
/* Device allocation outside any caching allocator (its base pointer can be
 * exported with cxs_ipc_get_handle). */
int cxs_device_alloc(size_t bytes, void** ptr);
int cxs_device_free(void* ptr);
/* Export / import a cxs_device_alloc allocation between processes (64-byte
 * handle); the import is mapped on the current device with peer access. */
int cxs_ipc_get_handle(const void* ptr, void* handle);
int cxs_ipc_open_handle(const void* handle, void** ptr);
int cxs_ipc_close(void* ptr);
/* One exchange step of rank `rank` out of `ranks` (at most 8): the step
 * number is *counter + 1 (device int32, updated in place); the kernel makes
 * this rank's earlier stores visible system-wide, writes the step into slot
 * `rank` of every peer's flag array (peer_flags[p], int32 [ranks], mapped
 * from that peer; entry `rank` itself is ignored) with release semantics,
 * then waits with acquire loads until every peer's slot in this rank's own
 * `flags` reaches the step, giving up after `spin_limit` clock cycles with
 * CXS_DEVICE_ERR_READY_TIMEOUT in `error`. Graph-capturable. */
int cxs_exchange_barrier(int32_t* counter, int32_t* const* peer_flags, int32_t* flags,
                         int32_t rank, int32_t ranks, int64_t spin_limit, int32_t* error,
                         void* stream);

/* -------------------------------------------- compressed branch + top-n ---
 * Compressed-token attention over complete summaries and top-n block
 * selection from the summed GQA probabilities (models/nsa/ops.py:73-123;
 * third_party/nsa_runtime/kernels.py:13-230). Selection order: current block
 * first, then score descending with ties to the lower block id; width =
 * min(count, ceil(total / BS)) with count <= 32 (the attend launch takes at
 * most 32 selected blocks per row); entries after the current block are -1.
 */
int cxs_compressed_select(const void* query,      /* [Q, H, 16, 64] bf16 */
                          const void* compressed, /* [C, H, 128] bf16 (K || V) */
                          int32_t summaries,      /* C */
                          const int32_t* positions, /* [Q] */
                          int32_t queries, int32_t heads, int32_t block_size,
                          int32_t count, int64_t total,
                          void* out,              /* [Q, H, 16, 64] bf16 */
                          int32_t* blocks,        /* [Q, H, width] */
                          float* scores,          /* [Q, H, C] or NULL */
                          void* stream);

/* cxs_compressed_select over candidate segments (segment_start and
 * segment_tokens as in cxs_attend_geometry, both multiples of block_size;
 * 0, 0 is cxs_compressed_select). Summaries use segment positions: summary c
 * covers positions [c * BS, (c + 1) * BS). A row of segment s skips the
 * summaries of the gap, selects among its visible blocks and returns
 * segment block ids; `total` is the true history + suffix length of one
 * candidate (it fixes width). No counterpart in the reference. */
int cxs_compressed_select_segments(const void* query, const void* compressed,
                                   int32_t summaries, const int32_t* positions,
                                   int32_t queries, int32_t heads, int32_t block_size,
                                   int32_t count, int64_t total, int64_t segment_start,
                                   int64_t segment_tokens, void* out, int32_t* blocks,
                                   float* scores, void* stream);

/* Compressed branch + top-n in the NSA paper's geometry (Yuan et al. 2025), of which the two
 * entry points above are the special case window = stride = block_size,
 * forced = 0. No counterpart in the reference. Compressed key i (row i of
 * `compressed`) summarises the tokens [i * stride, i * stride + window); a
 * row at true position p attends to the keys with i * stride + window <=
 * p + 1. Selection-block scores: block j sums, in ascending i, the key
 * scores of the windows overlapping it, each weighted by its stride steps
 * inside the block (the published NSA aggregation; the identity when window
 * = stride = block_size). Top-n: the current block, then with forced = 1
 * the block before it and block 0, then the other earlier blocks by score
 * descending, ties to the lower id.
 * With candidate segments (as in cxs_attend_geometry) key slots below
 * seg_key = (segment_start - window) / stride + 1 are the windows that end
 * in the shared history; candidate s owns segment_tokens / stride slots
 * after them, slot seg_key + s * (segment_tokens / stride) + k being true
 * window seg_key + k of that candidate (windows that cross segment_start
 * included). `scores` (optional) receives [Q, H, columns] block scores,
 * columns from cxs_select_score_columns. */
typedef struct cxs_select_geometry {
  int32_t queries, heads, block_size, count;
  int32_t summaries;  /* compressed keys C */
  int32_t window;     /* tokens per compressed key (a multiple of stride) */
  int32_t stride;     /* tokens between keys (divides block_size) */
  int32_t forced;     /* 1: previous and first block follow the current one */
  int64_t total;      /* true history + suffix length of one candidate */
  int64_t segment_start, segment_tokens;  /* 0, 0: one suffix */
} cxs_select_geometry;
int cxs_compressed_select_nsa(const cxs_select_geometry* geometry, const void* query,
                              const void* compressed, const int32_t* positions, void* out,
                              int32_t* blocks, float* scores, void* stream);
/* Columns of the block-score output of cxs_compressed_select_nsa. */
int cxs_select_score_columns(const cxs_select_geometry* geometry, int32_t* columns);

/* Mean-pool complete BS-token blocks of `tokens` records [n, H, 128] into
 * `summaries` [n / BS, H, 128] bf16 (models/nsa/ops.py:62-70). */
int cxs_block_summaries(const void* tokens, int64_t count, int32_t heads, int32_t block_size,
                        void* summaries, void* stream);
/* cxs_block_summaries for `segments` runs at once: run s pools the `count`
 * records starting at tokens + s * token_stride records into summaries +
 * s * summary_stride records (one launch for every candidate segment). */
int cxs_block_summaries_segments(const void* tokens, int64_t count, int32_t heads,
                                 int32_t block_size, void* summaries, int32_t segments,
                                 int64_t token_stride, int64_t summary_stride, void* stream);

/* ------------------------------------------------------- layer glue ---
 * Fused elementwise steps around the cuBLAS projections of one NSA layer,
 * keeping the reference's bf16 rounding sequence
 * (models/tensor_ops.py:6-26, models/nsa/model.py:440-492). */

/* out[r] = bf16(bf16(x[r] * rsqrt(mean(x[r]^2) + eps)) * weight), bf16 rows. */
int cxs_rms_norm(const void* x, const void* weight, void* out, int32_t rows, int32_t dim,
                 float eps, void* stream);

/* The residual add of a projection and the RMSNorm that follows it, in one
 * launch and in the reference's bf16 sequence (hidden = hidden + F.linear(..),
 * then rms_norm; models/nsa/model.py:440-492): hidden[r] = bf16(hidden[r] +
 * delta[r]) in place, out[r] = bf16(bf16(hidden[r] * rsqrt(mean(hidden[r]^2) +
 * eps)) * weight). Rows are 16-byte aligned, dim a multiple of 8. */
int cxs_residual_rms_norm(void* hidden, const void* delta, const void* weight, void* out,
                          int32_t rows, int32_t dim, float eps, void* stream);
/* From the fused projection [tokens, q_heads*64 | kv*64 (k) | kv*64 (v) | q_heads*3 (g)]
 * (row stride proj_stride elements): rotary q/k (rotate-half, inv_freq [32]),
 * write query [tokens, q_heads, 64], records [tokens, kv, 128] (K || V, row
 * stride records_stride), per-head current KV [kv][tokens, 128] (head stride
 * current_stride) and sigmoid gates [tokens, q_heads * 3]. */
int cxs_qkv_rope(const void* proj, int32_t proj_stride, const int32_t* positions,
                 const float* inv_freq, int32_t tokens, int32_t q_heads, int32_t kv_heads,
                 void* query, void* records, int32_t records_stride, void* current,
                 int32_t current_stride, void* gates, void* stream);
/* cxs_qkv_rope for candidate segments: token t writes its record and current
 * KV at row (t / segment_rows) * segment_stride + t % segment_rows instead of
 * row t (segment_rows = tokens per candidate, segment_stride = records per
 * candidate segment); query and gates stay at row t. */
int cxs_qkv_rope_segments(const void* proj, int32_t proj_stride, const int32_t* positions,
                          const float* inv_freq, int32_t tokens, int32_t q_heads,
                          int32_t kv_heads, void* query, void* records, int32_t records_stride,
                          void* current, int32_t current_stride, void* gates,
                          int32_t segment_rows, int32_t segment_stride, void* stream);
/* Keys of `windows` compressed windows (the NSA paper's MLP compression; no
 * counterpart in the reference): window i gathers the `window` (32)
 * records rows[i * window + t] of `records` [*, heads, 128] bf16 (K || V);
 * for K (part 0) and V (part 1) separately, x = bf16(records + pe[part])
 * ([window, 64]), key = bf16(W2[part] bf16(silu(bf16(W1[part] vec(x))))),
 * W1 [2, hidden, window * 64], W2 [2, 64, hidden] bf16, fp32 accumulation,
 * written to keys[slots[i]] ([*, heads, 128]). `scratch` holds
 * 2 * heads * windows * hidden fp32. Two launches. */
int cxs_compress_windows(const void* records, const int64_t* rows, int32_t windows,
                         int32_t heads, int32_t window, int32_t hidden, const void* pe,
                         const void* w1, const void* w2, void* scratch, void* keys,
                         const int64_t* slots, void* stream);
/* out[r, c] = bf16(silu(gate_up[r, c])) * gate_up[r, ffn + c] (SwiGLU). */
int cxs_silu_mul(const void* gate_up, int32_t rows, int32_t ffn, void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CXLSPARSE_B200_H */
