/* maivs_b200.h - C ABI of the B200 MAIVS query engine.
 *
 * One opaque handle is one FlatCellIndex. Every entry point below replaces one method of the
 * reference's Python/Rust API (src/index.rs #[pymethods], src/prof.rs), keeping its argument
 * meaning, defaults (in the comments) and error behaviour; each cites the reference line it
 * replaces. The index is built on the host cores; search runs on the GPU, and fails with
 * MAIVS_NO_DEVICE when no CUDA device is visible (there is no CPU fallback).
 *
 * All functions return a maivs_status. On failure maivs_last_error(handle) describes the cause.
 * Buffers are caller-owned, C-contiguous, and only read during the call.
 */
#ifndef MAIVS_B200_H
#define MAIVS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct maivs_index maivs_index;

typedef enum {
    MAIVS_OK = 0,
    MAIVS_BAD_SHAPE = 1,   /* dimension mismatch (PyValueError, index.rs:3329-3336) */
    MAIVS_BAD_ARG = 2,     /* invalid argument (e.g. scan_mode, index.rs:2683-2685) */
    MAIVS_BAD_STATE = 3,   /* e.g. add_batch before centroids (index.rs:2993-2996) */
    MAIVS_OOM = 4,         /* host or device allocation failed */
    MAIVS_CUDA_ERROR = 5,  /* a CUDA call failed */
    MAIVS_OVERFLOW = 6,    /* candidate buffers overflowed after enlarging them */
    MAIVS_UNSUPPORTED = 7, /* an option the GPU engine does not implement */
    MAIVS_NOT_FOUND = 8,   /* unknown id or array name */
    MAIVS_NO_DEVICE = 9    /* no CUDA device */
} maivs_status;

/* FlatCellIndex(dim, scan_mode="f32", rerank_factor=4, seed=0x5EED, code_bits=0)
 * (index.rs:2672-2755). Only scan_mode "binary" is served by the GPU search. */
int maivs_index_new(size_t dim, const char* scan_mode, size_t rerank_factor, uint64_t seed, size_t code_bits,
                    maivs_index** out);
void maivs_index_free(maivs_index* ix);
const char* maivs_last_error(const maivs_index* ix);
const char* maivs_status_string(int status);

/* train_centroids(vectors, n_cells, sample=262144, seed=0x5EED) (index.rs:2761-2804) */
int maivs_train_centroids(maivs_index* ix, const float* vectors, size_t n, size_t n_cells, size_t sample,
                          uint64_t seed);
/* set_centroids(centroids) (index.rs:2806-2821) */
int maivs_set_centroids(maivs_index* ix, const float* centroids, size_t m);
/* add_batch(ids, vectors) (index.rs:2987-3212) */
int maivs_add_batch(maivs_index* ix, const uint64_t* ids, const float* vectors, size_t n);
/* remove(id) -> bool (index.rs:3223-3276); *removed = 0 when the id is unknown */
int maivs_remove(maivs_index* ix, uint64_t id, int* removed);
/* compact() (index.rs:3565-3569) */
int maivs_compact(maivs_index* ix);

/* query-time and build-time switches (index.rs:2828-2984, :3520-3558) */
int maivs_set_rerank_factor(maivs_index* ix, size_t rf);                                      /* :2949 */
int maivs_set_two_stage(maivs_index* ix, int on, size_t mult);                                /* :2882 */
int maivs_set_tree_route(maivs_index* ix, int on, size_t min_cells, size_t fanout, float beam_frac); /* :2839 */
int maivs_set_graph_route(maivs_index* ix, int on, size_t min_cells);                         /* :2858 */
int maivs_set_adaptive(maivs_index* ix, int on, float margin);                                /* :2899 */
int maivs_set_fastscan(maivs_index* ix, int on);                                              /* :2962 */
int maivs_set_orthogonal_polysemy(maivs_index* ix, size_t homes, float lam);                  /* :2979 */
int maivs_set_replication(maivs_index* ix, size_t max_assign, float spill_margin);            /* :2970 */
int maivs_set_per_dim_sq(maivs_index* ix, int on);                                            /* :2908 */
int maivs_set_i8_rerank(maivs_index* ix, int on);                                             /* :2828 */
int maivs_set_centroid_sq8(maivs_index* ix, int on);                                          /* :2872 */
int maivs_set_tags(maivs_index* ix, const uint64_t* ids, const uint32_t* tags, size_t n);     /* :3535 */
/* set_filter(lo=None, hi=None): has_filter = 0 clears it (index.rs:3550-3558) */
int maivs_set_filter(maivs_index* ix, int has_filter, uint32_t lo, uint32_t hi);
/* Smallest batch that takes the cell-major join (the reference uses 2 x its thread pool,
 * index.rs:3348); default 32. */
int maivs_set_cell_major_min_batch(maivs_index* ix, size_t n);

/* Build device (no counterpart in the reference, which builds on its CPU threads): with
 * device >= 0, train_centroids, add_batch and the centroid tree run their k-means and their
 * vector placement on that GPU (exact-order dot products, so the index is the one the host build
 * makes, array for array); -1 (the default) builds on the host cores. A build step the GPU could
 * not run is computed on the host and counted in stats "build_gpu_failures". */
int maivs_set_build_device(maivs_index* ix, int device);

/* __len__ (index.rs:3474) */
int maivs_len(const maivs_index* ix, size_t* n);
/* One value of stats() (index.rs:3393-3472) by name, e.g. "n_cells", "tree_depth". */
int maivs_stat(maivs_index* ix, const char* name, double* value);

/* Build (or rebuild) the device image on CUDA device `device`. search* calls do this on their
 * first use (device 0, or the last one given) and after any mutation. */
int maivs_to_device(maivs_index* ix, int device);

/* search(query, k, nprobe=16, target_confidence=0.95, beta=8.0) (index.rs:3283-3305).
 * Writes up to k results, best first; *n_out = how many (no padding). */
int maivs_search(maivs_index* ix, const float* query, size_t k, size_t nprobe, float target_confidence, float beta,
                 uint64_t* ids, float* scores, size_t* n_out);

/* search_batch(queries, k, nprobe=16, target_confidence=0.95, beta=8.0, cell_major=True)
 * (index.rs:3316-3391). ids/scores are nq*k, row-major, padded with UINT64_MAX / -inf. A compacted
 * FastScan index is scanned by FastScan table sums (cell-major join or per query); any other index
 * (before compact(), after a remove(), FastScan off) by Hamming distance per query, as the reference
 * does (index.rs:1624-1626); the cell-major join of a compacted index without FastScan blocks is
 * MAIVS_UNSUPPORTED on the GPU (search it with cell_major = 0, or set FastScan and compact).
 * `queries` may be any host memory; queries in page-locked memory (cudaMallocHost, cudaHostRegister)
 * are copied to the device from where they are, others through the library's pinned staging buffer. */
int maivs_search_batch(maivs_index* ix, const float* queries, size_t nq, size_t k, size_t nprobe,
                       float target_confidence, float beta, int cell_major, uint64_t* ids, float* scores);

/* search_batch with device-resident queries and outputs, enqueued on `stream` (a cudaStream_t;
 * NULL = the handle's stream). Returns once the work is enqueued; after synchronising the stream,
 * maivs_device_flags() reports whether any query's candidate buffer overflowed (then the results
 * of that call must be discarded and the call repeated; the handle has already enlarged its
 * buffers). Same semantics as maivs_search_batch otherwise. Searches on one handle share its
 * workspace: a search enqueued on another stream than the handle's previous one waits for it on
 * the device (an event), so the two never overlap. */
int maivs_search_batch_device(maivs_index* ix, const float* d_queries, size_t nq, size_t k, size_t nprobe,
                              float target_confidence, float beta, int cell_major, uint64_t* d_ids, float* d_scores,
                              void* stream);
/* Overflow / routing-error counters of the last device search (synchronises `stream`); non-zero
 * means: search again (the candidate buffers have been enlarged). On a sharded handle the call is
 * collective and returns the sum over all ranks, so every rank takes the same decision. */
int maivs_device_flags(maivs_index* ix, void* stream, uint32_t* flags);

/* Allocation-free search (no counterpart in the reference). For callers that must not allocate
 * device memory while serving: a process whose GPU memory is already held by another runtime's
 * pool, or a latency-bound loop that cannot afford cudaMalloc's device-wide synchronisation.
 * Runs the per-query path (search_batch with cell_major = 0) on at most 64 device-resident
 * queries, enqueued on `stream`, with every intermediate buffer carved from one 32 MiB device
 * array that the library reserves statically on each GPU it uses. It allocates nothing:
 *  - the device image must be current (call maivs_to_device() after the last mutation), else
 *    MAIVS_BAD_STATE;
 *  - more than 64 queries, or a search whose buffers (about nq x nprobe x 1 KiB for 128-member
 *    cells) exceed 32 MiB, is rejected with MAIVS_BAD_ARG and a message giving the size;
 *  - the first call on a device looks the array's address up (a CUDA runtime call; under CUDA's
 *    lazy module loading that is also when the 32 MiB are reserved on that device), so make that
 *    call before capturing the stream into a graph. The address is kept per device ordinal: after
 *    a context reset (cudaDeviceReset) the next call does not look it up again, so a caller that
 *    resets a device must not use this entry point on it afterwards;
 *  - after the work completes, read maivs_device_flags(ix, stream, &f): non-zero means this
 *    call's ids and scores are invalid. Either a routing shortlist was longer than 16,384 cells
 *    (only with nprobe above 8,192: lower nprobe) or a bounded wait of the rerank ran out (the
 *    call may be repeated). Unlike maivs_search_batch_device, repeating the call enlarges
 *    nothing here; the array's size is fixed.
 * All calls, from every handle, share the one array. Nothing in it needs to start at zero, but
 * calls whose work overlaps on the GPU race on it: issue them on one stream or one at a time.
 * For every request it accepts, the results match maivs_search_batch_device(..., cell_major = 0,
 * ...) exactly. */
int maivs_search_batch_device_noalloc(maivs_index* ix, const float* d_queries, size_t nq, size_t k, size_t nprobe,
                                      float target_confidence, float beta, uint64_t* d_ids, float* d_scores,
                                      void* stream);

/* save(path) / load(path) (index.rs:3594-3603, src/persist.rs): the reference's on-disk format
 * "MAIVS2\0\1", so files move between the two implementations. A loaded index is not compacted
 * and has FastScan off, as in the reference, so it is searched per query by Hamming distance;
 * maivs_set_fastscan(1) and maivs_compact() give it the FastScan scan and the cell-major join.
 * maivs_load always returns a handle in *out (on failure it holds the
 * message for maivs_last_error; free it with maivs_index_free). Only scan_mode "binary" files
 * without f16 rerank rows load. */
int maivs_save(maivs_index* ix, const char* path);
int maivs_load(const char* path, maivs_index** out);

/* Cell-range sharding over the GPUs of one job (no counterpart in the reference, which runs in
 * one process; the cell-range split is its stated unit of parallelism, docs/ARCHITECTURE.md:28-30).
 * Rank r of `world` keeps the scan data of a contiguous range of cells holding ~1/world of the
 * member entries, plus the whole routing tables and rerank rows. Every search on a sharded handle
 * runs the cell-major join with three NCCL all-gathers (the seed cut-off, the candidate cut-off and
 * the best-k lists, merged on the device), so every rank must issue the same searches with the same
 * queries, and each rank's results equal the unsharded cell-major join's bit for bit.
 * maivs_nccl_unique_id: 128 bytes that rank 0 makes and the host sends to every rank.
 * maivs_shard: collective; world = 1 returns the handle to unsharded searching. NCCL is loaded
 * (libnccl.so.2) only here; a rank that does not join ends the set-up with an error after 120 s.
 * maivs_shard_range: the cells [lo, hi) of rank `rank` (host only).
 * maivs_search_batch_sharded_emulated: the same protocol with `world` shards inside this process on
 * the handle's device, exchanging through device copies (a one-GPU check of the sharded path; it
 * keeps `world` device images). */
int maivs_nccl_unique_id(uint8_t* id, size_t cap);
int maivs_shard(maivs_index* ix, int rank, int world, const uint8_t* nccl_id, size_t id_len);
int maivs_shard_range(maivs_index* ix, int rank, int world, uint32_t* lo, uint32_t* hi);
int maivs_search_batch_sharded_emulated(maivs_index* ix, int world, const float* d_queries, size_t nq, size_t k,
                                        size_t nprobe, float target_confidence, float beta, uint64_t* d_ids,
                                        float* d_scores, void* stream);

/* Host copy of one internal array, for persistence, inspection and parity tests: the pointer
 * stays valid until the next mutation of the index. Names: "vecs_f32", "scan_i8", "bits",
 * "ext_ids", "slot_cell", "slot_cells", "cell_members", "cell_member_off", "centroids",
 * "r_bound", "prim_len", "rep_off", "fs_codes", "fs_off", "cent_bits", "cent_sq8", "csq_min",
 * "csq_step", "sq_min", "sq_step", "signs", "tags", "tree_level_n", "tree_codes",
 * "tree_code_off", "tree_child_start", "tree_child_len", "tree_child_off", "tree_leaf_codes",
 * "tree_leaf_ids", "config". */
int maivs_array(maivs_index* ix, const char* name, const void** data, size_t* count, size_t* elem_bytes);

/* ConcurrentIndex (src/concurrent.rs): immutable sealed segments plus one mutable head, deletes
 * as tombstones by external id; reads never wait for a whole insert batch. One opaque handle is
 * one ConcurrentIndex. Inserts, deletes, sealing and the configuration run on the host cores under
 * the reference's locks (head -> sealed -> dead); search runs every segment and the head on the
 * GPU by the per-query path (Hamming scan: segments never have FastScan blocks, as fork_empty
 * turns FastScan off) and merges them in one kernel: tombstones dropped, one entry per id (its
 * best score), best k, exact score ties by ascending id. Calls on one handle may come from any
 * number of threads; its GPU searches run one at a time. Status codes as above;
 * maivs_concurrent_last_error describes the last failure. */
typedef struct maivs_concurrent maivs_concurrent;

/* ConcurrentIndex(dim, scan_mode="binary", rerank_factor=8, seed=0x5EED, code_bits=0,
 * seal_at=1000000) (concurrent.rs:159-172). On failure *out still holds a handle carrying the
 * message; free it with maivs_concurrent_free. */
int maivs_concurrent_new(size_t dim, const char* scan_mode, size_t rerank_factor, uint64_t seed, size_t code_bits,
                         size_t seal_at, maivs_concurrent** out);
void maivs_concurrent_free(maivs_concurrent* cx);
const char* maivs_concurrent_last_error(maivs_concurrent* cx);
/* train_centroids(vectors, n_cells, sample=262144, seed=0x5EED) on the head (concurrent.rs:322-326) */
int maivs_concurrent_train_centroids(maivs_concurrent* cx, const float* vectors, size_t n, size_t n_cells,
                                     size_t sample, uint64_t seed);
/* add_batch(ids, vectors) (concurrent.rs:247-261): into the head, which is compacted and sealed
 * into a segment once it holds seal_at vectors (the new head keeps its centroids, fork_empty). */
int maivs_concurrent_add_batch(maivs_concurrent* cx, const uint64_t* ids, const float* vectors, size_t n);
/* remove(id) -> bool (concurrent.rs:265-277): a tombstone; *removed = 0 for an unknown id or one
 * already removed. remove_many(ids) -> count (:280-293). */
int maivs_concurrent_remove(maivs_concurrent* cx, uint64_t id, int* removed);
int maivs_concurrent_remove_many(maivs_concurrent* cx, const uint64_t* ids, size_t n, size_t* n_removed);
/* seal() (:296-299); purge_head() -> count (:304-314): tombstoned head vectors are removed (in
 * ascending id; the reference walks a hash set) and the head compacted; compact() (:343). */
int maivs_concurrent_seal(maivs_concurrent* cx);
int maivs_concurrent_purge_head(maivs_concurrent* cx, size_t* n_purged);
int maivs_concurrent_compact(maivs_concurrent* cx);
/* head configuration (concurrent.rs:328-341); a sealed segment keeps the settings it was built
 * with. set_parallel_scan only records the flag: it picks the reference's CPU threading, and the
 * GPU scan is parallel either way (keeping every tie at the cut-off, as the sequential path). */
int maivs_concurrent_set_per_dim_sq(maivs_concurrent* cx, int on);
int maivs_concurrent_set_two_stage(maivs_concurrent* cx, int on, size_t mult);
int maivs_concurrent_set_adaptive(maivs_concurrent* cx, int on, float margin);
int maivs_concurrent_set_parallel_scan(maivs_concurrent* cx, int on);
int maivs_concurrent_set_graph_route(maivs_concurrent* cx, int on, size_t min_cells);
int maivs_concurrent_set_tree_route(maivs_concurrent* cx, int on, size_t min_cells, size_t fanout,
                                    float beam_frac);
/* Build device of the head and of every later head (no counterpart in the reference), as
 * maivs_set_build_device. */
int maivs_concurrent_set_build_device(maivs_concurrent* cx, int device);
/* __len__ (:219-224) and one value of stats() (:226-242): "segments", "head_live",
 * "sealed_live", "tombstones", "n_live", or any maivs_stat name of the head. */
int maivs_concurrent_len(maivs_concurrent* cx, size_t* n);
int maivs_concurrent_stat(maivs_concurrent* cx, const char* name, double* value);
/* CUDA device of the searches (default 0). */
int maivs_concurrent_to_device(maivs_concurrent* cx, int device);
/* search(query, k, nprobe=16, target_confidence=0.95, beta=8.0) (:176-185): up to k results,
 * *n_out of them. search_batch(queries, ...) (:187-217): nq*k, padded with UINT64_MAX / -inf. */
int maivs_concurrent_search(maivs_concurrent* cx, const float* query, size_t k, size_t nprobe,
                            float target_confidence, float beta, uint64_t* ids, float* scores, size_t* n_out);
int maivs_concurrent_search_batch(maivs_concurrent* cx, const float* queries, size_t nq, size_t k, size_t nprobe,
                                  float target_confidence, float beta, uint64_t* ids, float* scores);
/* Inspection (no counterpart in the reference): the number of sealed segments, and one array of
 * segment `segment` (-1 = the head) under maivs_array's names; the pointer stays valid until that
 * segment next changes. */
int maivs_concurrent_segments(maivs_concurrent* cx, size_t* n);
/* Instrumentation (no counterpart in the reference): per-kernel device times of this handle's
 * searches (every segment, the head and the merge), as maivs_kernel_clock / maivs_kernel_times. */
int maivs_concurrent_kernel_clock(maivs_concurrent* cx, int on);
int maivs_concurrent_kernel_times(maivs_concurrent* cx, int reset, const char** names, double* ms,
                                  uint64_t* launches, size_t cap, size_t* n_out);
int maivs_concurrent_array(maivs_concurrent* cx, long long segment, const char* name, const void** data,
                           size_t* count, size_t* elem_bytes);

/* profile(on) / profile_read(reset=True) (src/prof.rs:76-98): device time per query phase. The
 * reader fills up to `cap` (name, milliseconds) pairs; names are static strings. */
int maivs_profile(int on);
int maivs_profile_read(int reset, const char** names, double* values, size_t cap, size_t* n_out);

/* Instrumentation (no counterpart in the reference; used by bench.py and the profiles):
 * per-kernel device times while the clock is on, the number of kernels this library launched,
 * and the work counters of the last search ("nq", "probes", "candidates", "rerank_bytes",
 * "scan_code_bytes", "scan_pairs", ...; names '\n'-separated in `names`). */
int maivs_kernel_clock(maivs_index* ix, int on);
/* Times only the named kernel ("k_rerank", "k_seed", ... as maivs_kernel_times names them), so
 * that the events of the clock do not sit between every pair of kernels; NULL or "" times all.
 * Turns the clock on. MAIVS_BAD_ARG for an unknown name. */
int maivs_kernel_clock_only(maivs_index* ix, const char* kernel);
int maivs_kernel_times(maivs_index* ix, int reset, const char** names, double* ms, uint64_t* launches, size_t cap,
                       size_t* n_out);
/* Per kernel, the device time during which at least one of its launches ran, since the clock's
 * last reset (maivs_kernel_times with reset): launches on several streams that overlap in time
 * (the two halves of a split batch) count once here and once each in maivs_kernel_times. */
int maivs_kernel_busy(maivs_index* ix, const char** names, double* busy_ms, size_t cap, size_t* n_out);
uint64_t maivs_launch_count(void);
/* Host threads of the index build and host-side search staging for the calling thread
 * (omp_set_num_threads; no counterpart in the reference). Under launchers that export
 * OMP_NUM_THREADS=1 (torchrun) this restores the build's parallelism. MAIVS_BAD_ARG for n < 1. */
int maivs_set_num_threads(int n);
int maivs_last_search_stats(maivs_index* ix, char* names, size_t names_cap, double* values, size_t cap,
                            size_t* n_out);

/* Diagnostics (no counterpart in the reference): run one search (host buffers) only up to
 * `stage` and return its intermediate results - stage 0: query sign codes (nq x nw words),
 * FastScan tables (nq x 16*npos bytes), their delta and bias; stage 1: probe lists (nq x nprobe,
 * UINT32_MAX padded), re-order scores and counts; stage 2: the candidate slots sent to the exact
 * rerank, ascending (nq x cand_cap, UINT32_MAX padded) and their counts. Any output may be NULL. */
int maivs_debug_stage(maivs_index* ix, int stage, const float* queries, size_t nq, size_t k, size_t nprobe,
                      float target_confidence, float beta, int cell_major, uint64_t* qbits, uint8_t* lut,
                      float* delta, float* bias, uint32_t* chosen, float* cscore, uint32_t* nch, uint32_t* cand,
                      size_t cand_cap, uint32_t* cand_n);

/* Diagnostics: per-query internals of the cell-major join for one batch - seed survivors, seed
 * cut-off tau, end of the unpruned probe range, survivors of the scan - and the CUDA status. */
int maivs_debug_cellmajor(maivs_index* ix, const float* queries, size_t nq, size_t k, size_t nprobe,
                          float target_confidence, float beta, uint32_t* seed_n, uint32_t* tau, uint32_t* rest_hi,
                          uint32_t* rest_n, char* info, size_t info_cap);

#ifdef __cplusplus
}
#endif

#endif /* MAIVS_B200_H */
