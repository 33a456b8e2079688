/*
 * mak_kvcache.h — C ABI of the B200 (sm_100a) KV-cache movement and FP8
 * quantization library (libmak_kvcache.so).
 *
 * This is the drop-in native boundary for the `kvcache` operator family of
 * musa-aiter.  Every entry point takes plain device pointers, sizes and a
 * CUDA stream (`void*` holding a cudaStream_t; NULL = legacy default stream),
 * enqueues its kernels on that stream without synchronising, and returns
 * MAK_OK (0) or a negative MAK_E_* status.  `mak_last_error()` gives a
 * thread-local message for the last failing call on the calling thread.
 *
 * The library allocates no device memory.  Entry points that need scratch
 * memory (last-writer-wins resolution of duplicate destination slots) take a
 * caller-owned workspace whose size is given by `mak_scatter_workspace_bytes`,
 * or (the *_owned forms) a caller-kept owner table that persists across calls.
 *
 * Layout vocabulary (element strides unless stated otherwise):
 *   - "tile" caches keep block_size innermost: [L][NB][NH][HD][BS]
 *     (reference layout of musa_aiter/ops/kv_transfer.py:2987-3000);
 *   - "row" caches keep a token's hidden vector contiguous: [..][NB][BS][W]
 *     (LMCache, SGLang MP, MLA flat caches, DSV4 byte rows, HiCache pages).
 *
 * Each entry point names the reference launcher(s) it replaces.  Reference
 * paths are relative to the musa-aiter v0.5.0 source tree.
 */
#ifndef MAK_KVCACHE_H
#define MAK_KVCACHE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MAK_ABI_VERSION 1

#if defined(__GNUC__)
#define MAK_API __attribute__((visibility("default")))
#else
#define MAK_API
#endif

/* ---- status codes ------------------------------------------------------ */
#define MAK_OK 0
#define MAK_E_INVALID (-1)     /* bad shape, stride, pointer or argument */
#define MAK_E_UNSUPPORTED (-2) /* valid request this build does not handle */
#define MAK_E_WORKSPACE (-3)   /* workspace missing or too small */
#define MAK_E_CUDA (-4)        /* a CUDA runtime call or launch failed */

/* ---- element / index type codes ----------------------------------------- */
#define MAK_DT_U8 0
#define MAK_DT_F16 1
#define MAK_DT_BF16 2
#define MAK_DT_F32 3
#define MAK_DT_I32 4
#define MAK_DT_I64 5

/* ---- FP8 formats and scale modes ---------------------------------------- */
#define MAK_FP8_E4M3 1 /* 4 exponent bits, bias 7, finite max 480 (code 0x7F) */
#define MAK_FP8_E5M2 2 /* 5 exponent bits, bias 15, finite max 114688 */

#define MAK_SCALE_SCALAR 0         /* scale[0] */
#define MAK_SCALE_PER_HEAD 1       /* scale[h], h < num_heads */
#define MAK_SCALE_PER_LAYER_HEAD 2 /* scale[l * num_heads + h] */

/* Maximum planes (cache tensors) one row-family call may name. */
#define MAK_MAX_PLANES 4096

/*
 * Tile cache: element (l, b, h, d, o) of plane kv lives at
 *   k_or_v + l*stride_layer + b*stride_block + h*stride_head + d*stride_dim + o
 * (the block-offset stride is 1).  `v` may be NULL for single-plane calls.
 */
typedef struct mak_paged_desc {
  void* k;
  void* v;
  int64_t num_layers;
  int64_t num_blocks;
  int64_t num_heads;
  int64_t head_dim;
  int64_t block_size;
  int64_t stride_layer;
  int64_t stride_block;
  int64_t stride_head;
  int64_t stride_dim;
  int32_t dtype; /* MAK_DT_* of the stored elements (U8 for FP8 caches) */
  int32_t reserved;
} mak_paged_desc;

/*
 * Token-major linear buffer: element (l, t, h, d) of plane kv lives at
 *   k_or_v + l*stride_layer + t*stride_token + h*stride_head + d
 * (head_dim stride is 1).  Merged [T,2,NH,HD] buffers are two planes whose
 * pointers differ by NH*HD elements and whose stride_token is 2*NH*HD.
 */
typedef struct mak_linear_desc {
  void* k;
  void* v;
  int64_t num_tokens;
  int64_t stride_layer;
  int64_t stride_token;
  int64_t stride_head;
  int32_t dtype;
  int32_t reserved;
} mak_linear_desc;

/*
 * Row side: `num_planes` planes whose row r lives at
 *   plane_ptrs[p] + (r / rows_per_block)*block_stride + (r % rows_per_block)*row_stride
 * (strides in BYTES).  Rows r outside [0, num_rows) are skipped by the
 * kernels (never read or written), so a bad index cannot fault the GPU;
 * callers that must reject them validate first with `mak_slot_max`.
 * `plane_ptrs` is a HOST array of device addresses; `row_bytes` (host array,
 * may be NULL = all planes use `row_bytes0`) gives each plane's row width.
 */
typedef struct mak_rows_desc {
  const uint64_t* plane_ptrs;
  int64_t num_planes;
  int64_t rows_per_block;
  int64_t block_stride;
  int64_t row_stride;
  int64_t num_rows;
} mak_rows_desc;

/* ---- library probes ------------------------------------------------------ */

/* ABI version (replaces the *_abi_version getters,
 * csrc/kvcache/kv_transfer_float.mu:3021-3027, fp8_kv_cache.mu:1529,
 * hicache_transfer.mu:53). */
MAK_API int mak_abi_version(void);

/* Thread-local message of the last failing call on this thread. */
MAK_API const char* mak_last_error(void);

/* Number of SMs of the current device (cached per device). */
MAK_API int mak_device_sm_count(void);

/* Host-side count of kernels this library has launched since load (all
 * devices, all threads).  Used by benchmarks to report their launch count. */
MAK_API uint64_t mak_launch_count(void);

/* ---- plan builder --------------------------------------------------------- */

/*
 * Device reduction for slot validation: writes max(slots) (or -1 when every
 * slot is negative) to *out_max (device int64).  One launch; no sync.
 * Replaces the host-synchronising checks of musa_aiter/ops/kv_transfer.py:3020-3028.
 */
MAK_API int mak_slot_max(const void* slots, int32_t slot_dtype, int64_t n, int64_t* out_max, void* stream);

/* Bytes of workspace the scatter entry points need for `n_items` slots. */
MAK_API size_t mak_scatter_workspace_bytes(int64_t n_items);

/*
 * Last-writer-wins resolution: writes eff[i] = slots[i] when i is the last
 * index holding that slot value, else -1 (negative slots stay -1).  Uses the
 * workspace as an open-addressing hash table.  `eff` (int64, n entries) may
 * live inside the workspace tail (see mak_scatter_workspace_bytes).
 * Reference semantics: sequential token loop of musa_aiter/ops/kv_transfer.py:3092-3112.
 */
MAK_API int mak_resolve_last_writer(const void* slots, int32_t slot_dtype, int64_t n, int64_t* eff, void* workspace,
                            size_t workspace_bytes, void* stream);

/*
 * Dense slot mapping from block tables: for sequence b and position s < max_seq,
 *   slots[b*max_seq + s] = s < seq_lens[b] ? block_tables[b*bt_stride + s/block_size]*block_size + s%block_size : -1.
 * Replaces the per-sequence Python slot building of
 * musa_aiter/ops/kv_transfer.py:1779-1791 and the block-table walk of
 * csrc/kvcache/kv_transfer_float.mu:985-1164.
 */
MAK_API int mak_build_slot_mapping(const void* block_tables, int32_t bt_dtype, int64_t bt_stride, const void* seq_lens,
                           int32_t len_dtype, int64_t batch, int64_t max_seq, int64_t block_size, int64_t* slots,
                           void* stream);

/*
 * Dense slot vector from CSR-style token indices (SGLang Triton decode layout):
 *   slots[b*max_seq + s] = s < min(indptr[b+1] - indptr[b], max_seq) ? indices[indptr[b] + s] : -1.
 * Replaces the per-sequence index_select loop of musa_aiter/ops/kv_transfer.py:1291-1366
 * and musa_aiter_kv_triton_indexed_to_dense_* (csrc/kvcache/kv_transfer_float.mu:88-167).
 */
MAK_API int mak_build_indexed_slots(const void* indptr, int32_t indptr_dtype, const void* indices, int32_t indices_dtype,
                                    int64_t n_indices, int64_t batch, int64_t max_seq, int64_t* slots, void* stream);

/* ---- tile family ([L][NB][NH][HD][BS] caches) --------------------------- */

/*
 * Gather cache slots into token rows, every layer of `cache` in one launch.
 * fill_zero=1 writes zeros for negative slots ("zeros"), 0 leaves them
 * untouched ("preserve").  Slots >= NB*BS are skipped.
 * Replaces musa_aiter_kv_paged_to_linear_{float,half,bfloat16},
 * ..._multi_layer_*, ..._paged_to_merged_linear[_multi_layer]_*
 * (csrc/kvcache/kv_transfer_float.mu:16-86, 237-312, 387-671;
 *  lmcache_kv_transfer_extended.mu:241-401).
 */
MAK_API int mak_kv_paged_to_linear(const mak_paged_desc* cache, const mak_linear_desc* out, const void* slots,
                           int32_t slot_dtype, int32_t fill_zero, void* stream);

/*
 * Scatter token rows into cache slots (negative slots skipped, duplicate
 * slots: the last token wins).  Needs mak_scatter_workspace_bytes(T) bytes.
 * Replaces musa_aiter_kv_linear_to_paged_*, ..._multi_layer_*,
 * ..._merged_linear_to_paged[_multi_layer]_*
 * (csrc/kvcache/kv_transfer_float.mu:169-235, 314-385, 387-671).
 */
MAK_API int mak_kv_linear_to_paged(const mak_linear_desc* in, const mak_paged_desc* cache, const void* slots,
                           int32_t slot_dtype, void* workspace, size_t workspace_bytes, void* stream);

/*
 * FP8 gather + dequantize: out = decode(cache byte) * scale, rounded to the
 * output dtype (F16/BF16/F32); negative slots give zeros.
 * Replaces musa_aiter_kv_paged_fp8_to_linear_{e4m3,e5m2}, the vec4/hd*_bs*
 * variants and the multi-layer ones (csrc/kvcache/fp8_kv_cache.mu:183-272,
 * 363-452, 454-740, 742-1460).
 */
MAK_API int mak_kv_paged_fp8_to_linear(const mak_paged_desc* cache, const mak_linear_desc* out, const void* slots,
                               int32_t slot_dtype, const float* k_scale, const float* v_scale, int32_t scale_mode,
                               int32_t fp8_format, void* stream);

/*
 * FP8 quantize + scatter: byte = encode(x / scale) with the musa-aiter
 * reference encoder (round-half-even mantissa, flush below min-normal,
 * saturate to the format's largest finite code, non-finite -> signed zero).
 * Duplicate slots: the last token wins.
 * Replaces musa_aiter_kv_linear_to_paged_fp8_{e4m3,e5m2} and the vec4 and
 * multi-layer variants (csrc/kvcache/fp8_kv_cache.mu:146-272, 326-452,
 * 454-740, 742-882).
 */
MAK_API int mak_kv_linear_to_paged_fp8(const mak_linear_desc* in, const mak_paged_desc* cache, const void* slots,
                               int32_t slot_dtype, const float* k_scale, const float* v_scale, int32_t scale_mode,
                               int32_t fp8_format, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The four calls above with a segment map: a device vector of uint32 that the
 * pass over runs of consecutive slots fills with (epoch << 2) | (this window's
 * single-slot runs are left to the single-slot pass), one entry per window of
 * 8-32 tokens (ceil(T / 8) entries always suffice; a smaller map is ignored).
 * With a map, the run pass also moves the single slots of windows holding at
 * most four of them, and the single-slot pass skips the windows and slots the
 * map says it has nothing to do for, instead of scanning them.  epoch in
 * [1, 2^30) must differ from the one of any call still in flight on the same
 * map; entries of other epochs are never trusted, so a map may start with any
 * contents.  Calls of at most 512 tokens have no run pass and leave the map
 * untouched.  Results are identical to the unmapped calls.  Host-side
 * additions, no reference counterpart.
 */
MAK_API int mak_kv_paged_to_linear_mapped(const mak_paged_desc* cache, const mak_linear_desc* out, const void* slots,
                                          int32_t slot_dtype, int32_t fill_zero, uint32_t* seg_map,
                                          int64_t seg_map_entries, uint32_t epoch, void* stream);
MAK_API int mak_kv_linear_to_paged_mapped(const mak_linear_desc* in, const mak_paged_desc* cache, const void* slots,
                                          int32_t slot_dtype, void* workspace, size_t workspace_bytes,
                                          uint32_t* seg_map, int64_t seg_map_entries, uint32_t epoch, void* stream);
MAK_API int mak_kv_paged_fp8_to_linear_mapped(const mak_paged_desc* cache, const mak_linear_desc* out,
                                              const void* slots, int32_t slot_dtype, const float* k_scale,
                                              const float* v_scale, int32_t scale_mode, int32_t fp8_format,
                                              uint32_t* seg_map, int64_t seg_map_entries, uint32_t epoch,
                                              void* stream);
MAK_API int mak_kv_linear_to_paged_fp8_mapped(const mak_linear_desc* in, const mak_paged_desc* cache,
                                              const void* slots, int32_t slot_dtype, const float* k_scale,
                                              const float* v_scale, int32_t scale_mode, int32_t fp8_format,
                                              void* workspace, size_t workspace_bytes, uint32_t* seg_map,
                                              int64_t seg_map_entries, uint32_t epoch, void* stream);

/*
 * The two tile scatters with the owner-table last-writer resolution of
 * mak_rows_scatterv_owned (owner_rows >= num_blocks * block_size; same table,
 * epoch and zeroing rules) instead of a workspace, plus the optional segment
 * map of the *_mapped calls (seg_map may be NULL).  Results are identical to
 * mak_kv_linear_to_paged / mak_kv_linear_to_paged_fp8.  Host-side additions,
 * no reference counterpart.
 */
MAK_API int mak_kv_linear_to_paged_owned(const mak_linear_desc* in, const mak_paged_desc* cache, const void* slots,
                                         int32_t slot_dtype, uint64_t* owner, int64_t owner_rows, uint32_t epoch,
                                         uint32_t* seg_map, int64_t seg_map_entries, uint32_t seg_epoch,
                                         void* stream);
MAK_API int mak_kv_linear_to_paged_fp8_owned(const mak_linear_desc* in, const mak_paged_desc* cache,
                                             const void* slots, int32_t slot_dtype, const float* k_scale,
                                             const float* v_scale, int32_t scale_mode, int32_t fp8_format,
                                             uint64_t* owner, int64_t owner_rows, uint32_t epoch, uint32_t* seg_map,
                                             int64_t seg_map_entries, uint32_t seg_epoch, void* stream);

/* ---- row family (token-major caches) ------------------------------------ */

/*
 * Gather: for every plane p and token t < linear->num_rows,
 *   t < n_slots and slots[t] valid -> linear row t = paged row slots[t];
 *   otherwise (negative slot, out-of-range slot, or t >= n_slots) the linear
 *   row is zeroed when fill_zero=1 and left untouched when fill_zero=0.
 * paged and linear must name the same number of planes.
 * Replaces lmcache_paged_to_kv_buffer[_u16], ..._mla[_u16], ..._list_{u16,float},
 * ..._two_x_nl_{u16,float}, ..._two_x_nl_coalesced_u16, lmcache_mla_paged_to_buffer_list_*,
 * musa_aiter_kv_paged_to_mla_linear_* (csrc/kvcache/kv_transfer_float.mu:1592-1934,
 * 2032-2441, 673-826; lmcache_kv_transfer_extended.mu:7-239, 403-478).
 */
MAK_API int mak_rows_gather(const mak_rows_desc* paged, const mak_rows_desc* linear, const int64_t* row_bytes,
                    int64_t row_bytes0, const void* slots, int32_t slot_dtype, int64_t n_slots, int32_t fill_zero,
                    void* stream);

/*
 * Scatter: for every plane p and t < n_slots with slots[t] >= 0,
 *   paged row slots[t] = linear row (t + skip_prefix); duplicates: last t wins.
 * Needs mak_scatter_workspace_bytes(n_slots) bytes of workspace.
 * Replaces lmcache_kv_buffer_to_paged[_u16], ..._mla[_u16], ..._list_*,
 * ..._two_x_nl_*, lmcache_mla_buffer_to_paged_list_*, musa_aiter_kv_mla_linear_to_paged_*.
 */
MAK_API int mak_rows_scatter(const mak_rows_desc* linear, const mak_rows_desc* paged, const int64_t* row_bytes,
                     int64_t row_bytes0, const void* slots, int32_t slot_dtype, int64_t n_slots, int64_t skip_prefix,
                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * Grouped forms: `paged` and `linear` are arrays of n_groups (1..4)
 * descriptors; group g's planes follow group g-1's, and row_bytes (if not NULL)
 * gives one width per GROUP.  Lets planes of different geometry (e.g. the MLA
 * latent cache and its rope cache) move in one launch with one slot resolution.
 * Replaces the pair of per-cache launches the reference makes for MLA flat
 * caches (musa_aiter_kv_paged_to_mla_linear_* / musa_aiter_kv_mla_linear_to_paged_*,
 * csrc/kvcache/kv_transfer_float.mu:673-826, called twice from
 * ops/kv_transfer.py:3841-4118); same semantics as mak_rows_gather / mak_rows_scatter.
 */
MAK_API int mak_rows_gatherv(const mak_rows_desc* paged, const mak_rows_desc* linear, int32_t n_groups,
                             const int64_t* row_bytes, int64_t row_bytes0, const void* slots, int32_t slot_dtype,
                             int64_t n_slots, int32_t fill_zero, void* stream);
MAK_API int mak_rows_scatterv(const mak_rows_desc* linear, const mak_rows_desc* paged, int32_t n_groups,
                              const int64_t* row_bytes, int64_t row_bytes0, const void* slots, int32_t slot_dtype,
                              int64_t n_slots, int64_t skip_prefix, void* workspace, size_t workspace_bytes,
                              void* stream);

/*
 * mak_rows_scatterv with the last writer found through a caller-kept owner
 * table instead of the per-call workspace hash: one marking kernel sets
 * owner[slot] = max(owner[slot], epoch << 32 | token) and the copy moves a
 * token only while the entry still carries its own tag, so a scatter is two
 * launches (no memset, no resolve pass).  `owner` holds owner_rows uint64
 * entries in device memory (owner_rows >= every group's paged num_rows), is
 * zeroed once by the caller and then reused; every call on one table takes a
 * larger epoch than the calls before it (1 .. 2^32-1; after that zero the table
 * and restart at 1), and calls that share a table run in stream order (one
 * table per stream).  n_slots < 2^32.  Same results as mak_rows_scatterv
 * (reference semantics: musa_aiter/ops/kv_transfer.py:3092-3112, last token wins).
 */
MAK_API int mak_rows_scatterv_owned(const mak_rows_desc* linear, const mak_rows_desc* paged, int32_t n_groups,
                                    const int64_t* row_bytes, int64_t row_bytes0, const void* slots,
                                    int32_t slot_dtype, int64_t n_slots, int64_t skip_prefix, uint64_t* owner,
                                    int64_t owner_rows, uint32_t epoch, void* stream);

/*
 * Allocation-free row scatter.  No counterpart in the reference: it exists for
 * callers that cannot call cudaMalloc (a serving engine that reserved its HBM
 * up front and scatters inside its step loop, or a foreign-language caller
 * holding only raw pointers from another framework's allocator).  Same
 * semantics as mak_rows_scatter, but the duplicate-slot scratch lives in a
 * static device array inside the library (about 2.5 MiB on every GPU that
 * loads the library, held until exit), so no workspace is passed.
 * - At most MAK_STATIC_SCATTER_MAX_SLOTS slots per call; larger calls return
 *   MAK_E_UNSUPPORTED without launching anything.
 * - The first call on a device (per CUDA context: the primary context, or a
 *   driver-API context the caller made current) looks up the array's device
 *   address there; make that first call before any stream capture.  A device
 *   reset (cudaDeviceReset) after the first call is not supported.
 * - Every call shares the one array: calls that may overlap on the GPU (other
 *   streams, other host threads) race and must be serialised by the caller.
 * - Allocates nothing: no cudaMalloc, cudaFree or allocating library routine.
 */
#define MAK_STATIC_SCATTER_MAX_SLOTS 65536
MAK_API int mak_rows_scatter_static(const mak_rows_desc* linear, const mak_rows_desc* paged, const int64_t* row_bytes,
                                    int64_t row_bytes0, const void* slots, int32_t slot_dtype, int64_t n_slots,
                                    int64_t skip_prefix, void* stream);

/*
 * Indexed row copy: dst row dst_idx[i] = src row src_idx[i] for i < n, on
 * every plane pair.  A NULL index array means the identity (i).  Negative
 * indices on either side skip the item; rows out of range are skipped.  Duplicate destinations: the last i wins (needs workspace).
 * Replaces musa_aiter_kv_copy_paged_rows_{u8,layer_table_u8,contig_layers_u8}
 * (csrc/kvcache/kv_transfer_float.mu:3047-3279), musa_aiter_kv_copy_paged_blocks_*
 * and ..._fp8_vec8 (kv_transfer_float.mu:907-983, 1379; fp8_kv_cache.mu:1462-1527).
 */
MAK_API int mak_rows_copy(const mak_rows_desc* src, const mak_rows_desc* dst, const int64_t* row_bytes, int64_t row_bytes0,
                  const void* src_idx, int32_t src_idx_dtype, const void* dst_idx, int32_t dst_idx_dtype, int64_t n,
                  void* workspace, size_t workspace_bytes, void* stream);
/* mak_rows_copy with an indexed destination whose duplicate destinations are
 * resolved through a caller-kept owner table instead of a workspace (same table
 * and epoch rules as mak_rows_scatterv_owned; owner_rows >= dst->num_rows):
 * one marking launch, then the copy.  Same replaced launchers as mak_rows_copy. */
MAK_API int mak_rows_copy_owned(const mak_rows_desc* src, const mak_rows_desc* dst, const int64_t* row_bytes,
                                int64_t row_bytes0, const void* src_idx, int32_t src_idx_dtype, const void* dst_idx,
                                int32_t dst_idx_dtype, int64_t n, uint64_t* owner, int64_t owner_rows, uint32_t epoch,
                                void* stream);


/*
 * DSV4 MLA / blocked-scale staging <-> paged byte-block transfer: one launch
 * for every layer and block of a batch.  Arguments and semantics follow
 * lmcache_kv_strided_block_transfer (musa_aiter/ops/lmcache_kv_transfer.py:1294-1403,
 * csrc/kvcache/kv_transfer_float.mu:3281-3405): staging [NL][staging_tokens][row_bytes],
 * paged_ptrs a HOST array of NL device page bases, block_ids a DEVICE int64
 * vector; mode 0 plain rows, mode 1 values-then-scales per block (here
 * value_bytes + scale_bytes must equal row_bytes); direction 0 staging -> paged,
 * 1 paged -> staging.  Negative block ids are skipped.
 */
MAK_API int mak_lmcache_strided_block_transfer(void* staging, const uint64_t* paged_ptrs, const int64_t* block_ids,
                                               int64_t direction, int64_t num_layers, int64_t idx_start, int64_t n_valid,
                                               int64_t offset_in_object, int64_t staging_tokens, int64_t block_size,
                                               int64_t row_bytes, int64_t paged_block_stride, int64_t mode,
                                               int64_t value_bytes, int64_t scale_bytes, void* stream);

/* ---- host <-> device byte-copy batch --------------------------------------- */

typedef struct mak_copy_entry {
  uint64_t dst;  /* destination address (device, or pinned host) */
  uint64_t src;  /* source address (device, or pinned host) */
  uint64_t size; /* bytes */
} mak_copy_entry;

#define MAK_COPY_AUTO 0   /* copy engine for entries >= engine_threshold, one kernel for the rest */
#define MAK_COPY_ENGINE 1 /* every entry on the copy engines (SMs stay free for compute) */
#define MAK_COPY_KERNEL 2 /* every entry through the batch-copy kernel */

/*
 * Submit a batch of byte copies on one stream, in order, without synchronising.
 * Host sides must be pinned (the kernel addresses them through unified
 * addressing); engine_threshold <= 0 means 4 MiB.  Replaces the MUSA
 * batched-copy submission of csrc/kvcache/lmcache_musa_batch_copy_ext.cpp:208-259
 * (no batched-memcpy runtime call is used: small entries are batched into
 * kernel launches of up to 128 entries instead).
 */
MAK_API int mak_memcpy_batch(const mak_copy_entry* entries, int64_t n, int32_t mode, int64_t engine_threshold,
                             void* stream);

/* CUDA runtime and driver versions the library sees (lmcache_musa_batch_copy_ext.cpp:177-206). */
MAK_API int mak_runtime_versions(int32_t* runtime_version, int32_t* driver_version);

/* ---- CacheGen-style codec ------------------------------------------------ */

/*
 * min and max of a float tensor (f16/bf16/f32, n > 0) into out_minmax[0..1]
 * (device float[2]); device-only, no host sync.
 */
MAK_API int mak_minmax(const void* x, int32_t dtype, int64_t n, float* out_minmax, void* stream);

/*
 * Uniform-bin encode with the reference's arithmetic (musa_aiter/ops/kv_transfer.py:1111-1172):
 * scale = (1 / (max - min)) * (num_bins - 1) in fp32, code = clamp(round_half_even((x - min) * scale)),
 * counts[num_bins] (device uint64) = histogram of the codes, cdf[num_bins + 1]
 * (device float) = [0, cumsum(counts) / n] accumulated sequentially in fp32.
 * minmax is the device output of mak_minmax.  Replaces musa_aiter_kv_cachegen_encode_float
 * (csrc/kvcache/kv_transfer_float.mu:828-866) and the host bincount.
 */
MAK_API int mak_cachegen_encode(const void* x, int32_t dtype, int64_t n, const float* minmax, int32_t num_bins,
                                uint8_t* codes, uint64_t* counts, float* cdf, void* stream);

/*
 * The encode's codebook on the device from mak_minmax's output: the reference builds it with
 * torch.linspace(min, max, num_bins) in float32 on the tensor's device, or fills it with min when
 * max == min (musa_aiter/ops/kv_transfer.py:1130-1132, 1147, 1167).  For a CUDA device that is
 * step = (max - min) / (num_bins - 1), then min + step * i (fused) for i < num_bins / 2 and
 * max - step * (num_bins - 1 - i) (fused) for the rest: bit-identical to torch.linspace on the GPU,
 * and no read-back of min / max to the host.  codebook: device float[num_bins].
 */
MAK_API int mak_cachegen_codebook(const float* minmax, int32_t num_bins, float* codebook, void* stream);

/* out[i] = codebook[codes[i]] converted to out_dtype (RNE).  Replaces
 * musa_aiter_kv_cachegen_decode_float (csrc/kvcache/kv_transfer_float.mu:868-905). */
MAK_API int mak_cachegen_decode(const uint8_t* codes, int64_t n, const void* codebook, int32_t codebook_dtype,
                                int32_t num_bins, void* out, int32_t out_dtype, void* stream);

/* ---- MLA FP8 rows with per-group scales ----------------------------------- */

/*
 * MLA latent + rope token rows of one or more layers:
 *   kv[l][t][0..kv_dim)  and  pe[l][t][0..pe_dim), element strides given,
 *   innermost stride 1, dtype MAK_DT_F16 or MAK_DT_BF16 (both tensors).
 */
typedef struct mak_mla_linear_desc {
  void* kv;
  void* pe;
  int64_t num_layers;
  int64_t num_tokens;
  int64_t kv_dim;          /* 256, 512 or 1024: groups of 128 */
  int64_t pe_dim;          /* multiple of 8, at most 256 */
  int64_t kv_stride_layer; /* elements */
  int64_t kv_stride_token;
  int64_t pe_stride_layer;
  int64_t pe_stride_token;
  int32_t dtype;
  int32_t reserved;
} mak_mla_linear_desc;

/*
 * FP8 MLA cache row, one per token and layer (the DeepSeek MLA FP8 row):
 *   [kv_dim FP8 codes][kv_dim/128 fp32 group scales][pe_dim rope elements, input dtype]
 * e.g. 512 + 16 + 128 = 656 bytes.  Group g's scale is the amax of the finite
 * |x| among its 128 values / fp8_max in fp32 (fp8_max 448 for E4M3, 57344 for
 * E5M2), so every stored scale is finite,
 * and each value is encoded with the musa-aiter FP8 rule as x / scale
 * (musa_aiter/ops/kv_transfer.py:2161-2183; an all-zero group stores scale 0 and
 * zero codes).  No reference counterpart: the reference only moves such rows as
 * opaque bytes (kv_copy_paged_rows_layer_table, ops/kv_transfer.py:4588-4616;
 * lmcache_kv_strided_block_transfer mode 1).  `cache` has one plane per layer,
 * row width mak_mla_fp8_row_bytes(kv_dim, pe_dim).
 *
 * store: quantise and scatter, last writer wins for duplicate slots, negative or
 *        out-of-range slots skipped; workspace = mak_scatter_workspace_bytes(n).
 * load:  gather and dequantise (code * scale, RNE to the output dtype); rows of
 *        negative or out-of-range slots become zeros.
 */
MAK_API int64_t mak_mla_fp8_row_bytes(int64_t kv_dim, int64_t pe_dim);
MAK_API int mak_mla_fp8_rows_store(const mak_mla_linear_desc* lin, const mak_rows_desc* cache, const void* slots,
                                   int32_t slot_dtype, int32_t fp8_format, void* workspace, size_t workspace_bytes,
                                   void* stream);
MAK_API int mak_mla_fp8_rows_load(const mak_rows_desc* cache, const mak_mla_linear_desc* lin, const void* slots,
                                  int32_t slot_dtype, int32_t fp8_format, void* stream);
/* store with the owner-table last-writer resolution of mak_rows_scatterv_owned
 * (owner_rows >= cache->num_rows; same table and epoch rules). */
MAK_API int mak_mla_fp8_rows_store_owned(const mak_mla_linear_desc* lin, const mak_rows_desc* cache,
                                         const void* slots, int32_t slot_dtype, int32_t fp8_format, uint64_t* owner,
                                         int64_t owner_rows, uint32_t epoch, void* stream);

/*
 * Self-check of the store's division-free quotient (a reciprocal per group and
 * Markstein's correction step per value, then the range-bounded encoder) against
 * the IEEE fp32 division and the full encoder on this device: for the 2^23
 * scales 2^scale_exp * [1, 2) and every 16-bit input of elem_dtype
 * (MAK_DT_BF16 / MAK_DT_F16) that a group with that scale can hold (|x / s| up
 * to fp8_max, inf and nan), adds to counts[0] the FP8 codes that differ and to
 * counts[1] the finite quotients >= 2^-14 in magnitude that differ in any bit
 * (device memory, 2 x uint64, zeroed by the caller).  Scales outside the fast range ([2^-60, 2^16]) take
 * the IEEE division in the store and are not counted.  Every call also checks
 * the group scale of the two-token store (amax / fp8_max by one multiply and a
 * correction step) against the IEEE division for every finite non-negative
 * 16-bit amax, adding differences to counts[1].  No reference counterpart: a
 * test entry point.
 */
MAK_API int mak_fp8_quotient_selfcheck(int32_t elem_dtype, int32_t fp8_format, int32_t scale_exp, uint64_t* counts,
                                       void* stream);

/* ---- rotary position embedding (the `cache` family) ----------------------- */

/*
 * Dtype codes: x_dtype / cos_dtype / sin_dtype are the operands; prod1_dtype is
 * the promoted type of (x, cos), prod2_dtype of (x, sin), sum_dtype of the two
 * products (torch type promotion; the caller computes them); out_dtype the
 * result.  f16 / bf16 steps round to nearest-even after every operation.
 */
typedef struct mak_rope_dense_desc {
  const void* x;
  const void* cos;        /* broadcast to the output's leading dims by strides (0 = broadcast) */
  const void* sin;
  void* out;              /* contiguous [rows, 2 * half] */
  int64_t rows;           /* product of the leading sizes */
  int64_t half;           /* head_dim / 2 */
  int64_t sizes[6];       /* leading sizes (ndim of them) */
  int64_t x_strides[7];   /* leading strides, then [6] = stride along head_dim (elements) */
  int64_t cos_strides[7]; /* leading strides, then [6] = stride along half */
  int64_t sin_strides[7];
  int32_t ndim;
  int32_t interleaved;    /* 1: pairs (2j, 2j+1); 0: pairs (j, j + half) */
  int32_t x_dtype, cos_dtype, sin_dtype, prod1_dtype, prod2_dtype, sum_dtype, out_dtype;
  int32_t reserved;
} mak_rope_dense_desc;

/* out = rope(x, cos, sin).  Replaces apply_rope (musa_aiter/ops/cache.py:9-42). */
MAK_API int mak_rope_dense(const mak_rope_dense_desc* desc, void* stream);

typedef struct mak_rope_cache_desc {
  void* cache;            /* key cache [num_blocks][num_heads][head_dim][block_size], rotated in place */
  const void* cos;        /* [max_positions, half] (row stride) or [half] (cos_stride_row = 0) */
  const void* sin;
  const void* slots;      /* per token; negative = skip */
  const void* positions;  /* per token, row of cos / sin */
  int64_t n_tokens;
  int64_t num_blocks, num_heads, head_dim, block_size;
  int64_t stride_block, stride_head, stride_dim; /* elements; block offset stride 1 */
  int64_t cos_stride_row, cos_stride_last, sin_stride_row, sin_stride_last;
  int32_t slot_dtype, pos_dtype;
  int32_t cache_dtype, cos_dtype, sin_dtype, prod1_dtype, prod2_dtype, sum_dtype;
  int32_t interleaved;
  int32_t reserved;
} mak_rope_cache_desc;

/*
 * Rotate key_cache[block, :, :, offset] of every token in place with the cos /
 * sin row of its position.  Slots must be distinct within one call (the caller
 * splits repeated slots into successive calls, which keeps the reference's
 * token order).  Tokens with a negative slot or position, or a block past
 * num_blocks, are skipped; positions must lie inside the cos / sin table.
 * Replaces apply_rope_to_key_cache (musa_aiter/ops/cache.py:45-102).
 */
MAK_API int mak_rope_key_cache(const mak_rope_cache_desc* desc, void* stream);

/* ---- peer mappings for block migration between GPUs of one node ----------- */

/*
 * No reference counterpart (the reference's communication layer raises for
 * world_size != 1, musa_aiter/communication.py:55-56).  A receiving process
 * exports a device pointer as the CUDA IPC handle of its allocation plus the
 * offset inside it; the sending process imports it (opened once per handle and
 * device, reference-counted) and moves blocks with mak_rows_copy, whose stores
 * then land in the peer's memory.  mak_ipc_release drops one import.
 * Handles are mak_ipc_handle_bytes() (64) bytes.
 */
MAK_API int mak_ipc_handle_bytes(void);
MAK_API int mak_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out);
MAK_API int mak_ipc_import(const void* handle, int64_t offset, void** ptr_out);
MAK_API int mak_ipc_release(const void* handle);

#ifdef __cplusplus
}
#endif

#endif /* MAK_KVCACHE_H */
