/*
 * libsabah_rt.so - the C ABI of the sm_100a routed-expert runtime.
 *
 * A drop-in for the reference runtime of Fovane/Sabah-MoE-Accelerator. Each
 * declaration names the reference export it replaces (file:line inside that
 * project). Conventions kept from the reference:
 *   - int-returning calls give 0 on success and -1 on failure, with the reason
 *     in sabah_rt_last_error() (one process-wide buffer, last failure wins,
 *     not thread-safe) - sabah/runtime/cuda/sabah_rt.cu:802-806, 3041;
 *   - pointer-returning calls give NULL on failure;
 *   - one device per process, chosen by sabah_rt_init.
 * Plain pointers and sizes only; no framework types cross this boundary.
 */
#ifndef SABAH_RT_H
#define SABAH_RT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- runtime ------------------------------------------------------------ */

/* Last error message. Ref sabah_rt.cu:3041. */
const char *sabah_rt_last_error(void);
/* cudaSetDevice(device), create the copy and compute streams, reset the
 * residency table and size the hot-tier slab from SABAH_LLAMA_HOT_BYTES
 * (default 2 GiB). Ref sabah_rt.cu:3190-3199. */
int sabah_rt_init(int device);
/* Drain both streams, release the slab, residency, scratch and pinned pool.
 * Ref sabah_rt.cu:3221-3232. */
int sabah_rt_shutdown(void);
/* Number of visible CUDA devices, 0 on error. Ref sabah_rt.cu:3234-3238. */
int sabah_rt_device_count(void);
/* "sabah_rt abi=v2 sentinel=N". Ref sabah_rt.cu:3839-3843. */
const char *sabah_rt_build_info(void);

/* ---- the hot path ---------------------------------------------------------- */

/* ggml MUL_MAT_ID over one expert tensor:
 *   dst[t][i][r] = sum_c W[ids[t][i]][r][c] * x[t][i % x_rows][c]
 * All strides are in bytes. source is the expert tensor [k, rows, n_experts]
 * (expert_stride = nb2, row_stride = nb1) of ggml type qt; x, ids, dst are
 * device memory; x_rows is 1 (broadcast) or n_ids (one input row per slot);
 * k % 32 == 0; an id outside [0, n_experts) is an error; n_tokens == 0 is a
 * counted no-op; stream NULL -> the runtime's compute stream; ids_key is an
 * opaque identity of the ids tensor that lets up to four consecutive calls on
 * the same ids skip the download (NULL: always download).
 * source in HOST memory (the llama.cpp contract): experts are made resident in
 * the hot-tier slab, keyed by (source, expert), after a download of the ids.
 * source in DEVICE memory (extension): the bank is read in place and the ids
 * never leave the device; an out-of-range id is then reported by the next call
 * (or sabah_rt_device_error) and its output slot is NaN.
 * Ref sabah_rt.cu:3494-3833; caller patches/llama.cpp/0001-sabah-native-mul-mat-id.patch:193-200. */
int sabah_rt_mul_mat_id_v2(const void *source, size_t expert_stride, size_t row_stride,
                           const void *d_x, size_t x_id_stride, int x_rows, size_t x_token_stride,
                           const void *d_ids, size_t ids_id_stride, size_t ids_token_stride, int n_ids,
                           int n_tokens, float *d_dst, size_t dst_id_stride, size_t dst_token_stride, int rows,
                           int k, int n_experts, int qt, void *stream, const void *ids_key);

/* One routed MoE block for one token on the compute stream:
 *   h[e][j] = silu(<Wg[e][j], x>) * <Wu[e][j], x>
 *   out[i]  = (accumulate ? out[i] : 0) + sum_e w[e] * <Wd[e][i], h[e]>
 * d_ptrs is a device array [gate x n_used, up x n_used, down x n_used] of
 * expert bases, d_w the routing weights, d_h scratch of n_used * ff floats.
 * Ref sabah_rt.cu:3362-3378 (kernels :2725-2785). */
int sabah_moe_block(const float *d_x, float *d_out, float *d_h, const void *const *d_ptrs, const float *d_w,
                    int d_model, int ff, int n_used, int qt_gate, int qt_up, int qt_down, int accumulate);

/* Extension of sabah_moe_block: n_tokens tokens, experts read in place from
 * device-resident banks [n_experts][rows][row bytes] with the router ids on the
 * device (ids and w are [n_tokens][n_used], x and out [n_tokens][d_model], h
 * [n_tokens][n_used][ff]). stream NULL -> compute stream. New in this build; it
 * replaces the pointer-table upload of the reference path (executor.py:61-99). */
int sabah_moe_block_ids(const void *gate_bank, const void *up_bank, const void *down_bank,
                        size_t gu_expert_stride, size_t down_expert_stride, int n_experts, const int32_t *d_ids,
                        const float *d_w, const float *d_x, float *d_out, float *d_h, int d_model, int ff,
                        int n_used, int n_tokens, int qt_gate, int qt_up, int qt_down, int accumulate,
                        void *stream);

/* sabah_moe_block_ids over gathered inputs. No reference counterpart.
 * Token t's input is row d_xrows[t] of d_x, which has n_xrows rows of d_model
 * floats; everything else is as sabah_moe_block_ids. The expert-parallel bank
 * (sharded experts, one process per GPU) calls it with the all-gathered
 * activations and, per local (token, slot) pair, the pair's token row, so no
 * separate gather pass runs. A row index outside [0, n_xrows) gives NaN
 * outputs for that token and the device error (sabah_rt_device_error). */
int sabah_moe_block_gather(const void *gate_bank, const void *up_bank, const void *down_bank,
                           size_t gu_expert_stride, size_t down_expert_stride, int n_experts, const int32_t *d_ids,
                           const float *d_w, const float *d_x, const int32_t *d_xrows, int n_xrows, float *d_out,
                           float *d_h, int d_model, int ff, int n_used, int n_tokens, int qt_gate, int qt_up,
                           int qt_down, int accumulate, void *stream);

/* sabah_moe_block_ids without any allocation. No reference counterpart.
 * sabah_moe_block_ids grows its cross-CTA scratch with cudaMalloc the first
 * time it meets a larger shape; this entry point never allocates device or
 * host memory, for a process whose device memory is carved up before serving
 * starts, or a caller holding a lock that the implicit device synchronization
 * of an allocation could deadlock on.
 * IQ3_S gate, up and down only, d_model and ff in {768, 1024, 1536, 2048}.
 * Its scratch is a fixed 1 MiB device array: n_tokens * n_used *
 * (2 * ff + d_model) * 4 bytes must fit in 960 KiB (e.g. 4 tokens x top-10 at
 * 2048/768), else -1 with the limit in sabah_rt_last_error().
 * Every call queues a clear of the array's arrival counters on its stream
 * (a memset, no allocation) ahead of its kernels; the first call on a device
 * (with that device current) also looks up the array's address. Calls share
 * the array, so calls that overlap on the GPU (two streams, two threads) race
 * and give wrong results. */
int sabah_moe_block_ids_noalloc(const void *gate_bank, const void *up_bank, const void *down_bank,
                                size_t gu_expert_stride, size_t down_expert_stride, int n_experts,
                                const int32_t *d_ids, const float *d_w, const float *d_x, float *d_out, float *d_h,
                                int d_model, int ff, int n_used, int n_tokens, int qt_gate, int qt_up, int qt_down,
                                int accumulate, void *stream);

/* n_layers routed blocks back to back on one stream with a residual update in
 * place: x <- x + block_L(x) for L = 0..n_layers-1. gate/up/down_banks are HOST
 * arrays of n_layers device pointers; ids/w are [n_layers][n_tokens][n_used] on
 * the device; h is [n_tokens][n_used][ff] scratch. New in this build: one call
 * per decoded token in place of the harness's per-block loop (executor.py:101-112). */
int sabah_moe_decode(int n_layers, const void *const *gate_banks, const void *const *up_banks,
                     const void *const *down_banks, size_t gu_expert_stride, size_t down_expert_stride,
                     int n_experts, const int32_t *d_ids, const float *d_w, float *d_x, float *d_h, int d_model,
                     int ff, int n_used, int n_tokens, int qt_gate, int qt_up, int qt_down, void *stream);

/* Reads and clears the device error word: 1 when a kernel reading a
 * device-resident bank met an expert id outside [0, n_experts), else 0.
 * New in this build (the device-resident path has no synchronous id check). */
int sabah_rt_device_error(void);

/* ---- dequantization ---------------------------------------------------------- */

/* Dequantize n elements (whole blocks) of type qt on the host, bit-exact with
 * gguf-py's dequantize. Ref sabah_rt.cu:3845-3847 (sb_host_dequant :2233-2423);
 * Q6_K (14) is added. */
int sabah_rt_host_dequant(const void *src, float *dst, int qt, int n);
/* Dequantize n_rows rows of row_elems elements on the device through the
 * kernels' own decoders; synchronous. Ref sabah_rt.cu:3879-3885. */
int sabah_dequant(const void *d_src, float *d_dst, int qt, int n_rows, int row_elems);
/* Bytes of one row of n elements of type qt, 0 if unsupported. Ref sabah_rt.cu:3887. */
size_t sabah_row_bytes(int qt, int n);

/* ---- counters ---------------------------------------------------------------- */

/* Counters as one JSON object (keys of ref sabah_rt.cu:3389-3413, plus
 * device_calls and id_reuse). Returns the snprintf length. Ref sabah_rt.cu:3835-3837. */
int sabah_rt_snapshot(char *buf, size_t n);
/* Ref sabah_rt.cu:3849-3862. */
int sabah_rt_get_diag(unsigned long long *calls, unsigned long long *tokens, unsigned long long *overflow,
                      unsigned long long *verify_ok, unsigned long long *verify_fail);
/* Ref sabah_rt.cu:3864-3877. */
int sabah_rt_get_metrics(unsigned long long *hits, unsigned long long *misses, unsigned long long *evictions,
                         unsigned long long *bytes_fetched, unsigned long long *resident_bytes);

/* Per-kernel device timing: every launch bracketed by a CUDA event pair on its
 * own stream (the reference's SABAH_LLAMA_EVENTS probe, sabah_rt.cu:3771-3825;
 * also on when SABAH_LLAMA_EVENTS=1). Switching clears the totals. */
int sabah_rt_kernel_timing(int on);
/* Totals since timing was switched on: {"kernel": [launches, ms], ...}. Waits
 * for the timed launches. Returns the snprintf length. */
int sabah_rt_kernel_times(char *buf, size_t n);

/* ---- hot-tier slab ------------------------------------------------------------- */

/* One cudaMalloc carved by best fit with coalescing frees. Ref sabah_rt.cu:3889-3901
 * (allocator :342-424). */
int sabah_slab_init(size_t capacity_bytes);
void *sabah_slab_alloc(size_t bytes);
void sabah_slab_free(void *ptr);
void sabah_slab_destroy(void);

/* ---- memory, copies, events (Python harness plumbing) ---------------------------- */

/* Ref sabah_rt.cu:3240-3245. */
void *sabah_dev_alloc(size_t bytes);
void sabah_dev_free(void *p);
/* Pooled pinned host blocks, reused and released at shutdown. Ref sabah_rt.cu:3250-3280. */
void *sabah_host_alloc(size_t bytes);
void sabah_host_free(void *p);
/* Ref sabah_rt.cu:3284-3291. */
int sabah_host_register(void *ptr, size_t bytes);
int sabah_host_unregister(void *ptr);
/* Ref sabah_rt.cu:3293-3305. */
int sabah_dev_mem(size_t *free_bytes, size_t *total_bytes);
int sabah_memcpy_h2d(void *dst, const void *src, size_t n);
int sabah_memcpy_d2h(void *dst, const void *src, size_t n);
int sabah_memset_d(void *dst, int v, size_t n);
/* H2D on the copy stream. Ref sabah_rt.cu:3308-3311. */
int sabah_h2d_async(void *dst, const void *src, size_t n);
/* Ref sabah_rt.cu:3313-3353. */
void *sabah_event_create(void);
void sabah_event_destroy(void *ev);
int sabah_event_record_copy(void *ev);
int sabah_event_record_compute(void *ev);
int sabah_compute_wait_event(void *ev);
int sabah_copy_wait_event(void *ev);
float sabah_event_elapsed_ms(void *a, void *b);
int sabah_event_sync(void *ev);
/* 1 complete, 0 in flight, -1 error. */
int sabah_event_query(void *ev);
int sabah_sync_copy(void);
int sabah_sync_compute(void);
int sabah_sync_all(void);

/* ---- file probes (Linux) ---------------------------------------------------------- */

/* Which file and offset a host pointer maps (via /proc/self/maps); registers
 * the file for sabah_rt_read_probe. Ref sabah_rt.cu:3046-3066 (Win32 there). */
int sabah_rt_resolve_probe(void *ptr, char *buf, size_t n);
/* O_DIRECT read of `bytes` at `off` of the first registered file; reports the
 * first 8 bytes. Ref sabah_rt.cu:3068-3094. */
int sabah_rt_read_probe(uint64_t off, size_t bytes, char *buf, size_t n);

/* ---- synthetic banks (benchmarks and tests) ------------------------------------------ */

/* Fill d_dst with n_rows dense rows of k elements of type qt (Q8_0, Q4_K, Q6_K,
 * IQ3_S) encoding N(0, sigma) weights drawn from `seed`; asynchronous on stream.
 * New in this build (the reference reads real GGUF files only). */
int sabah_synth_rows(void *d_dst, int qt, long long n_rows, int k, unsigned long long seed, float sigma,
                     void *stream);
/* Rows [row0, row0 + n_rows) of the same tensor (the same bytes a full
 * sabah_synth_rows call writes there), for one rank's slice of a sharded bank. */
int sabah_synth_rows_at(void *d_dst, int qt, long long row0, long long n_rows, int k, unsigned long long seed,
                        float sigma, void *stream);

/* ---- expert-parallel bank (rows of fp32 activations) -------------------------------- */

/* New in this build, for the expert-sharded bank (the reference has one GPU).
 * dst[i] = src[rows[i]] for i < n; rows of k floats (k % 4 == 0, 16-byte
 * aligned); an index outside [0, n_src) gives a zero row. Asynchronous. */
int sabah_ep_gather_rows(const float *d_src, int n_src, const int32_t *d_rows, int n, int k, float *d_dst,
                         void *stream);
/* dst[t] = sum of src rows offsets[t] .. offsets[t + 1] - 1 in increasing order
 * (deterministic), for t < n_out; offsets are clamped to [0, n_src]. Asynchronous. */
int sabah_ep_sum_rows(const float *d_src, int n_src, const int32_t *d_offsets, int n_out, int k, float *d_dst,
                      void *stream);
/* x += y over n floats (n % 4 == 0, 16-byte aligned). Asynchronous. */
int sabah_ep_add(float *d_x, const float *d_y, long long n, void *stream);
/* The layer's pair sums with the residual folded in:
 * dst[t] = (init_row0 <= t < init_row0 + n_init ? init[t - init_row0] : 0)
 *          + sum over i in [offsets[t], offsets[t + 1]) of src[idx ? idx[i] : i],
 * in increasing i (deterministic); a source index outside [0, n_src) adds
 * nothing. init may be dst itself (each element is read before it is
 * written); src must not overlap dst. Asynchronous. */
int sabah_ep_sum_rows_ex(const float *d_src, int n_src, const int32_t *d_idx, const int32_t *d_offsets, int n_out,
                         int k, float *d_dst, const float *d_init, int init_row0, int n_init, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SABAH_RT_H */
