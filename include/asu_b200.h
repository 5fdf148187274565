/*
 * asu_b200.h -- C ABI of the B200 KV-resolver hot path (libasu_b200.so).
 *
 * Plain pointers and sizes only; every pointer argument named as a tensor is
 * a CUDA device pointer (or, for host_pool, a device-accessible pointer to
 * mapped pinned host memory).  Every launch is asynchronous on `stream`
 * (a cudaStream_t; NULL = legacy default stream).
 *
 * Return value of every entry point: ASU_OK (0), a negative ASU_ERR_* for a
 * rejected argument (nothing was launched), or ASU_ERR_CUDA_BASE + cudaError_t
 * when the launch failed.  The reference launchers return void; an int is
 * ABI-compatible for callers that ignore the result (its ctypes harnesses set
 * restype themselves, ops/scripts/asu_hbm_index_common.py:283-316).
 *
 * Kernels never trap.  Where a `status` pointer is accepted it points to one
 * int32 per request row, and the kernel ORs ASU_ST_* bits into it; the
 * reference-named *_do launchers take no status word (their reference
 * signatures have none) and skip offending elements silently.
 *
 * Concurrency: no two launches may touch the same request row at the same
 * time (pta-ops/asu_hbm_index_lookup_simt/README.md:144-146).
 */
#ifndef ASU_B200_H
#define ASU_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes ---------------------------------------------------- */
#define ASU_OK 0
#define ASU_ERR_ARG (-1)          /* null pointer or size outside the supported range */
#define ASU_ERR_ALIGN (-2)        /* pointer / row size alignment a vector path requires */
#define ASU_ERR_CUDA_BASE 1000    /* ASU_ERR_CUDA_BASE + cudaError_t */

/* ---- device status bits (OR-ed per request row) ----------------------- */
#define ASU_ST_BAD_QUERY 0x01       /* a query id outside [0, key space) was skipped */
#define ASU_ST_FREE_EXHAUSTED 0x02  /* free list / stack ran out (reference: reads past it / raises) */
#define ASU_ST_RING_EXHAUSTED 0x04  /* maintain found fewer evictable slots than free_head (reference spins forever) */
#define ASU_ST_BAD_STATE 0x08       /* a map entry pointed outside its table (corrupt state) */
#define ASU_ST_SHORTAGE 0x10        /* LRU: some misses found no free slot (counted, not an error) */
#define ASU_ST_BAD_SOURCE 0x20      /* swap-in / resolver: source row out of range */
#define ASU_ST_BAD_TOKEN_STATE 0x40 /* resolver: token_state not in {ASU_ONLY, HBM_RESIDENT, TAIL_HBM} */
#define ASU_ST_NO_VICTIM 0x80       /* batch-LRU: more unique misses than evictable slots (state left unchanged) */
#define ASU_ST_TIMEOUT 0x100        /* swap-in: a bulk copy did not complete within its wait limit (rows skipped);
                                       a late copy may still land in shared memory, so the stream's later
                                       results are not to be trusted: handle it like a context error */

/* ---- reference constants (ops/asu_hbm_index_lookup_aiv.cpp:7-12) ------- */
#define ASU_HBM_INDEX_SIZE (128u * 1024u)
#define ASU_HBM_SLOT_COUNT (10u * 1024u)
#define ASU_HBM_FREE_SLOT_COUNT (2u * 1024u)
#define ASU_HBM_QUERY_COUNT (2u * 1024u)
#define ASU_HBM_QUERY_TILE 64u /* simu/hbm_lookup_update/src/hbm_lookup_update_kernel.cpp:7 */

/* LRU statistics columns (int64 per request row, accumulated with +=). */
#define ASU_LRU_STAT_HITS 0
#define ASU_LRU_STAT_MISSES 1
#define ASU_LRU_STAT_INSTALLS 2
#define ASU_LRU_STAT_SHORTAGES 3
#define ASU_LRU_STAT_EVICTIONS 4
#define ASU_LRU_STAT_COLS 5

/* Resolver token states (patch/0001 vllm_ascend/ops/asu_kv_resolver.py, patch lines 834-837). */
#define ASU_TOKEN_INVALID (-1)
#define ASU_TOKEN_ASU_ONLY 0
#define ASU_TOKEN_HBM_RESIDENT 1
#define ASU_TOKEN_TAIL_HBM 2

int asu_version(void);
const char* asu_status_string(int code);

/* ======================================================================
 * ops contract: lookup with sequential free-list allocation
 * ==================================================================== */

/* Replaces asu_hbm_index_lookup_do, ops/asu_hbm_index_lookup_aiv.cpp:170-189 (the same op is
 * aclnnAsuHbmIndexLookup behind ascend-ops/asu_hbm_index_lookup/asu_hbm_index_lookup_torch_adpt.h:15-39).
 * Fixed reference sizes: index [reqNum,128K], slotToIndex [reqNum,10K], freeSlots [reqNum,2K],
 * freeHead [reqNum], queryIndex / slotOut [reqNum,2K], all int32.  blockDim is advisory. */
int asu_hbm_index_lookup_do(uint32_t blockDim, void* stream, void* index, void* slotToIndex, void* freeSlots,
                            void* freeHead, void* queryIndex, void* slotOut, uint32_t reqNum);

/* Sized form of asu_hbm_index_lookup_do with a per-request status word (nullable). */
int asu_hbm_index_lookup_ex(void* stream, int32_t* index, int32_t* slot_to_index, const int32_t* free_slots,
                            int32_t* free_head, const int32_t* query_index, int32_t* slot_out, uint32_t req_num,
                            uint32_t index_size, uint32_t slot_count, uint32_t free_slot_count,
                            uint32_t query_count, int32_t* status);

/* ======================================================================
 * ops contract: hash-seeded ring maintain (eviction + free-list refill)
 * ==================================================================== */

/* Replaces asu_hbm_index_maintain_do, ops/asu_hbm_index_maintain_aicpu.cpp:15-38 (kernel
 * ops/asu_hbm_index_maintain_aicpu_kernel.aicpu:53-95; aclnnAsuHbmIndexMaintain behind
 * ascend-ops/asu_hbm_index_maintain/asu_hbm_index_maintain_torch_adpt.h:15-42).
 * lastQuerySlots [reqNum,2K] int32; reference sizes as above. */
int asu_hbm_index_maintain_do(uint32_t blockDim, void* stream, void* index, void* slotToIndex, void* freeSlots,
                              void* freeHead, void* lastQuerySlots, uint32_t reqNum, uint32_t seed);

int asu_hbm_index_maintain_ex(void* stream, int32_t* index, int32_t* slot_to_index, int32_t* free_slots,
                              int32_t* free_head, const int32_t* last_query_slots, uint32_t req_num, uint32_t seed,
                              uint32_t index_size, uint32_t slot_count, uint32_t free_slot_count,
                              uint32_t query_count, int32_t* status);

/* ======================================================================
 * pure gather + random update (simu/hbm_lookup_update)
 * ==================================================================== */

/* Replaces hbm_lookup_vec_do, simu/hbm_lookup_update/src/hbm_lookup_update_kernel.cpp:258-273.
 * tableStates [reqNum,128K]; queryKeys [reqNum,queryLen]; statesOut [reqNum, align64(queryLen)]
 * (the reference's padded layout; pad entries are written 0).  tableKeys and notFound are
 * accepted and ignored exactly as in the reference. */
int hbm_lookup_vec_do(uint32_t blockDim, void* stream, void* tableKeys, void* tableStates, void* queryKeys,
                      void* statesOut, uint32_t reqNum, uint32_t queryLen, int32_t notFound);

/* Replaces hbm_random_update_do, simu/hbm_lookup_update/src/hbm_lookup_update_kernel.cpp:275-292:
 * table[r, query[r,pos_t]] = newStates[r,pos_t] for t < floor(queryLen*updatePercent/100),
 * pos_t = (a*t + b) mod queryLen, later t winning on duplicate keys. */
int hbm_random_update_do(uint32_t blockDim, void* stream, void* tableKeys, void* tableStates, void* queryKeys,
                         void* newStates, uint32_t reqNum, uint32_t queryLen, uint32_t seed,
                         uint32_t updatePercent);

/* Sized gather: out[r*out_stride + i] = table[r*index_size + query[r*query_len + i]] for
 * i < query_len, 0 for query_len <= i < out_stride; hit_mask[r*query_len+i] = out != not_found
 * (nullable).  A key outside [0,index_size) yields not_found and ASU_ST_BAD_QUERY. */
int asu_gather_lookup(void* stream, const int32_t* table, uint32_t index_size, const int32_t* query,
                      uint32_t query_len, int32_t* out, uint32_t out_stride, uint8_t* hit_mask, uint32_t req_num,
                      int32_t not_found, int32_t* status);

int asu_random_update(void* stream, int32_t* table, uint32_t index_size, const int32_t* query,
                      const int32_t* new_states, uint32_t query_len, uint32_t req_num, uint32_t seed,
                      uint32_t update_percent, int32_t* status);

/* ======================================================================
 * batch-LRU lookup (Ascend 950 SIMT contract)
 * ==================================================================== */

/* Replaces asu_hbm_index_lookup_simt_do, pta-ops/asu_hbm_index_lookup_simt/include/
 * asu_hbm_index_lookup_simt_constants.h:19-27 (kernel src/asu_hbm_index_lookup_simt_kernel.cpp:10-271).
 * token_to_slot [req,128K] i32, slot_to_token [req,10K] i32, lru_slots [req,10K] i16,
 * query_token_ids / slot_ids [req,2K] i32, miss_mask [req,2K] u8 (bool).  `workspace` is
 * accepted for ABI compatibility and not used: all scratch lives in shared memory. */
int asu_hbm_index_lookup_simt_do(void* stream, void* token_to_slot, void* slot_to_token, void* lru_slots,
                                 void* query_token_ids, void* slot_ids, void* miss_mask, void* workspace,
                                 uint32_t req_num);

int asu_hbm_index_lookup_simt_ex(void* stream, int32_t* token_to_slot, int32_t* slot_to_token, int16_t* lru_slots,
                                 const int32_t* query_token_ids, int32_t* slot_ids, uint8_t* miss_mask,
                                 uint32_t req_num, uint32_t index_size, uint32_t slot_count, uint32_t query_count,
                                 int32_t* status);

/* ======================================================================
 * exact LRU slot pool: step-boundary maintain + resolve, one pool per request
 * ==================================================================== */

/* One decode step of LRUManagedCache (simu/kv_cache_eviction_sim.py:124-150) for every request row:
 *   1. evict LRU residents until free_count >= min(free_target, slot_count), pushing each
 *      victim slot on the free stack in eviction order; evicted keys -> evicted[r, :n];
 *   2. resolve query[r, :] in order: a resident key is a hit (moves to MRU), a miss pops the
 *      free stack (top first), or is a shortage (slot -1) when the stack is empty.
 * State per request row r (int32): token_to_slot [key_space] (-1 = absent), slot_to_token
 * [slot_count], lru_order [slot_count] (first slot_count - free_count entries: resident slots,
 * LRU first), free_stack [slot_count] (first free_count entries, top last), free_count.
 * Outputs: slot_out [Q], hit_mask [Q] (the simulator's per-query hit), install_mask [Q] (this
 * position took a slot and owes one swap-in), evicted [evicted_stride], evicted_count,
 * stats [ASU_LRU_STAT_COLS] int64 (+=, nullable), status (nullable).
 * Limits: slot_count <= 16384, query_count <= 4096, key_space < 2^31. */
int asu_lru_step(void* stream, int32_t* token_to_slot, int32_t* slot_to_token, int32_t* lru_order,
                 int32_t* free_stack, int32_t* free_count, const int32_t* query, int32_t* slot_out,
                 uint8_t* hit_mask, uint8_t* install_mask, int32_t* evicted, uint32_t evicted_stride,
                 int32_t* evicted_count, int64_t* stats, int32_t* status, uint32_t req_num, uint32_t key_space,
                 uint32_t slot_count, uint32_t query_count, uint32_t free_target);

/* asu_lru_step for a caller whose top-k is in pinned host memory (no reference counterpart: the
 * reference's top-k comes from the indexer on the NPU).  `query` is the device address of the
 * pinned, mapped [req_num, query_count] buffer (asu_host_device_pointer): the step reads it over
 * the host link itself instead of after an upload, and stores every query to query_copy
 * [req_num, query_count] in HBM, the copy a following asu_swapin_gather reads.  Everything else
 * as asu_lru_step. */
int asu_lru_step_host_query(void* stream, int32_t* token_to_slot, int32_t* slot_to_token, int32_t* lru_order,
                            int32_t* free_stack, int32_t* free_count, const int32_t* query, int32_t* query_copy,
                            int32_t* slot_out, uint8_t* hit_mask, uint8_t* install_mask, int32_t* evicted,
                            uint32_t evicted_stride, int32_t* evicted_count, int64_t* stats, int32_t* status,
                            uint32_t req_num, uint32_t key_space, uint32_t slot_count, uint32_t query_count,
                            uint32_t free_target);

/* ======================================================================
 * swap-in gather: host row pool -> HBM slot pool
 * ==================================================================== */

/* For every (r, pos) with install_mask set: copy row record_addr[r*key_space + query[r,pos]] of
 * host_pool (pool_rows rows of row_bytes bytes, consecutive rows host_pitch bytes apart, 0 =
 * row_bytes; device-accessible mapped pinned memory) into slot_pool[r, slot[r,pos]]
 * ([req, slot_count, row_bytes], HBM).  Replaces the MicroKV batch_get + H2D of the v0.1 design
 * (docs/v0.1/kv-cache-offload-v0.1-real-ops-design.md:293-312).  row_bytes and host_pitch must
 * be multiples of 16 and both pools 16-byte aligned.  Rows up to 1 KiB move as one TMA bulk copy
 * each (a host_pitch that is a multiple of 128 reads whole lines); a bulk copy that does not
 * complete within its wait limit sets ASU_ST_TIMEOUT and its lane stops. */
int asu_swapin_gather(void* stream, const void* host_pool, int64_t pool_rows, uint32_t row_bytes,
                      uint32_t host_pitch, const int32_t* record_addr, uint32_t key_space, const int32_t* query,
                      const int32_t* slot,
                      const uint8_t* install_mask, uint32_t query_count, void* slot_pool, uint32_t slot_count,
                      uint32_t req_num, int32_t* status);

/* Producer side of the swap-in: host_pool[dst_row ? dst_row[i] : i] = src[src_index ? src_index[i]
 * : i] for i < n (rows of row_bytes; src rows src_pitch bytes apart in device memory, host rows
 * host_pitch bytes apart, 0 = row_bytes); dst_row[i] < 0 skips item i.  A host row's padding
 * (host_pitch - row_bytes) under 128 bytes is written with zeros too.  Replaces the MicroKV
 * batch_put of prefilled records (docs/v0.1/kv-cache-offload-v0.1-real-ops-design.md:243-292;
 * MicroKV/python/microkv/client.py batch_put).  Out-of-range rows set ASU_ST_BAD_STATE (host
 * row) or ASU_ST_BAD_SOURCE (source row) in status[0] (nullable) and are skipped.  row_bytes and
 * both pitches must be multiples of 16, both pointers 16-byte aligned, and n * row_bytes / 16
 * below 2^31 (split larger write-backs). */
int asu_host_pool_writeback(void* stream, void* host_pool, int64_t pool_rows, uint32_t row_bytes,
                            uint32_t host_pitch, const void* src, int64_t src_rows, uint64_t src_pitch,
                            const int32_t* src_index, const int32_t* dst_row, int64_t n, int32_t* status);

/* Pinned, mapped host allocation for the row pool (cudaHostAlloc Portable|Mapped). */
int asu_host_pool_alloc(uint64_t bytes, void** host_ptr, void** device_ptr);
int asu_host_pool_free(void* host_ptr);

/* Device address of page-locked, mapped host memory (any pinned allocation, e.g. a torch pinned
 * tensor); fails for memory the GPU cannot address, so a kernel is never handed such a pointer.
 * Used to let kernels read their inputs from and write their outputs to host buffers directly. */
int asu_host_device_pointer(const void* host_ptr, void** device_ptr);

/* No reference counterpart (the reference's top-k and resolved slots stay on the NPU).  Copies
 * `bytes` from src to dst with the SMs, where one side is HBM and the other page-locked, mapped
 * host memory given by its device address (asu_host_device_pointer), or both are HBM: a host
 * <-> device transfer that does not use a copy engine, for a caller's small per-step uploads and
 * read-backs on a box whose copy engines share the host unevenly.  16-, 4- or 1-byte units by the
 * alignment of both pointers and the size; the ranges must not overlap (ASU_ERR_ARG).
 * Asynchronous on `stream`, a programmatic dependent launch. */
int asu_mapped_copy(void* stream, void* dst, const void* src, uint64_t bytes);

/* Self-test of the bounded device wait that asu_swapin_gather's TMA copies use (no reference
 * counterpart).  One thread waits on an mbarrier with an arrival count of one: arrive == 0 gives
 * a barrier nothing arrives at, so the wait runs out and ASU_ST_TIMEOUT is OR-ed
 * into status[0] (after ~1 s on B200: 2^18 tries); arrive != 0 arrives first and leaves
 * status[0] unchanged.  Asynchronous on
 * `stream`; the kernel returns either way and the context stays usable. */
int asu_selftest_bounded_wait(void* stream, int32_t arrive, int32_t* status);

/* ---- swap-in balancing across the GPUs of one box -------------------------
 * No reference counterpart: the reference's swap-in is a per-request MicroKV socket fetch on one
 * NPU (docs/v0.1/kv-cache-offload-v0.1-real-ops-design.md:293-312).  On a box whose GPUs share
 * the host memory system unevenly, a rank on a fast host link swaps in part of a slow rank's rows:
 * it reads them from the slow rank's host pool over its own link and stores them into the slow
 * rank's slot pool over NVLink. */

/* asu_swapin_gather with a slot pool in ANOTHER GPU's memory (peer_slot_pool: a CUDA IPC mapping
 * opened with asu_ipc_open, device peer access over NVLink).  Same arguments and status bits; rows
 * are written with plain 16-byte stores (no bulk or multicast copy touches the peer), and every
 * thread fences at system scope before the grid completes, so work ordered after this launch (an
 * event or a NCCL message the peer waits on) sees the rows. */
int asu_swapin_gather_to_peer(void* stream, const void* host_pool, int64_t pool_rows, uint32_t row_bytes,
                              uint32_t host_pitch, const int32_t* record_addr, uint32_t key_space,
                              const int32_t* query, const int32_t* slot, const uint8_t* install_mask,
                              uint32_t query_count, void* peer_slot_pool, uint32_t slot_count, uint32_t req_num,
                              int32_t* status);

/* Page-lock and map existing host memory (e.g. another process's pool mapped from a shared-memory
 * file descriptor) for this process's CUDA context: cudaHostRegister(Portable|Mapped). */
int asu_host_register(void* host_ptr, uint64_t bytes, void** device_ptr);
int asu_host_unregister(void* host_ptr);

/* CUDA IPC of a device allocation: `handle` (64 bytes) names the allocation that contains
 * device_ptr, `offset` is device_ptr's distance from its start.  asu_ipc_open maps it into the
 * calling process on the current device (peer access enabled lazily) and returns the mapping's
 * base; asu_ipc_close unmaps it. */
int asu_ipc_export(const void* device_ptr, uint8_t* handle, uint64_t* offset);
int asu_ipc_open(const uint8_t* handle, void** base_ptr);
int asu_ipc_close(void* base_ptr);

/* ======================================================================
 * single-request KV resolver (patch 0001 asu_kv_resolver custom op)
 * ==================================================================== */

/* Replaces aclnnAsuKvResolver behind npu_asu_resolve_kv_slots_single_req
 * (patch/0001 csrc/asu_kv_resolver/asu_kv_resolver_torch_adpt.h, patch lines 21-59; kernel
 * op_kernel/asu_kv_resolver.cpp, patch lines 394-452; schema patch lines 810-826).
 * Serial semantics over topk[0..topk_numel): HBM_RESIDENT -> hbm_slot_of_token; ASU_ONLY /
 * TAIL_HBM -> pop free_slot_stack[--free_slot_count], copy the KV row pair from source row
 * (asu_record_addr[tok], or block_table[tok/block_size]*block_size + tok%block_size) to the
 * popped managed slot, then mark resident.  kv rows are raw bytes (kv*_row_bytes each,
 * kv0_row_bytes + kv1_row_bytes <= 1 MiB; row pairs of up to 1280 bytes with 16-byte-aligned
 * starts are copied by the resolve launch itself, larger ones by a second launch).  The resolve
 * launch is a programmatic dependent launch: stream order holds for everything it reads and
 * writes.  On return `workspace` holds the install list:
 * int32 count, then (source row, managed slot) pairs in install order.
 * `workspace` must hold asu_kv_resolver_workspace_bytes(topk_numel) bytes of device memory.
 * status: one int32 (nullable). */
int asu_kv_resolver_do(void* stream, const int32_t* topk, int64_t topk_numel, int32_t* token_state,
                       const int32_t* asu_record_addr, int32_t* hbm_slot_of_token, int32_t* slot_owner_token,
                       const int32_t* free_slot_stack, int32_t* free_slot_count, int64_t free_slot_stack_len,
                       const int32_t* block_table, int64_t block_table_len, const void* kv0_src, const void* kv1_src,
                       void* kv0_dst, void* kv1_dst, int64_t kv0_row_bytes, int64_t kv1_row_bytes, int64_t src_rows,
                       int64_t slot_count, int64_t max_seq_len, int64_t actual_seq_len, int64_t block_size,
                       int32_t* resolved, void* workspace, int32_t* status);

int64_t asu_kv_resolver_workspace_bytes(int64_t topk_numel);

/* Replaces ASULayerKVCacheContext.reset_state (patch/0003 asu_kv_cache_manager.py, patch lines
 * 234-292) with one launch: token_state / asu_record_addr / hbm_slot_of_token [max_seq_len] and
 * slot_owner_token [slot_count] reset to INVALID, free_slot_stack = 0..slot_count-1,
 * free_slot_count = slot_count; positions below managed_prefix_len become ASU_ONLY with
 * record block_table[p/block_size]*block_size + p%block_size, positions up to actual_seq_len
 * TAIL_HBM.  Rejects (ASU_ERR_ARG) the lengths the reference raises on. */
int asu_resolver_reset(void* stream, int32_t* token_state, int32_t* asu_record_addr, int32_t* hbm_slot_of_token,
                       int64_t max_seq_len, int32_t* slot_owner_token, int32_t* free_slot_stack,
                       int32_t* free_slot_count, int64_t slot_count, const int32_t* block_table,
                       int64_t block_table_len, int64_t block_size, int64_t actual_seq_len,
                       int64_t managed_prefix_len);

/* The resolver over a bounded managed pool: asu_kv_resolver_do's token-state machine fused with
 * exact-LRU eviction, for a managed cache smaller than the context (e.g. 8192 resident + 2048
 * free slots at a 128K-token context).  No single reference function: it composes the resolver
 * (patch/0001 asu_kv_resolver.py, patch lines 954-1039), which raises "free_slot_stack does not
 * have enough slots" (patch lines 879-888) once the pool is full, with LRUManagedCache
 * (simu/kv_cache_eviction_sim.py:124-150):
 *   1. while free_slot_count < min(free_target, slot_count) and slots are resident, the least
 *      recently used slot (lru_order[0]) is evicted: its token returns to ASU_ONLY when
 *      asu_record_addr[tok] >= 0, else TAIL_HBM; hbm_slot_of_token[tok] and the slot's owner
 *      become INVALID; the slot is pushed on free_slot_stack;
 *   2. topk is resolved in order as by asu_kv_resolver_do, hits moving their slot to the most
 *      recently used end and installs entering there.
 * lru_order [slot_count] int32: the first slot_count - free_slot_count entries are the resident
 * slots, least recently used first (after asu_resolver_reset: none).  free_slot_stack,
 * slot_owner_token and lru_order all hold slot_count entries.  Limits: topk_numel <= 4096,
 * slot_count <= 16384, kv0_row_bytes + kv1_row_bytes <= 1 MiB; one launch, no workspace.
 * Differences from the reference on bad input: an entry whose source row is out of range sets
 * ASU_ST_BAD_SOURCE and takes no slot; no free slot left sets ASU_ST_FREE_EXHAUSTED (slot -1).
 * evicted (>= min(free_target, slot_count) entries) / evicted_count: the evicted tokens in
 * eviction order (both nullable); stats: ASU_LRU_STAT_COLS int64, += (nullable); status: one
 * int32 (nullable). */
int asu_kv_resolver_lru(void* stream, const int32_t* topk, int64_t topk_numel, int32_t* token_state,
                        const int32_t* asu_record_addr, int32_t* hbm_slot_of_token, int32_t* slot_owner_token,
                        int32_t* free_slot_stack, int32_t* free_slot_count, int32_t* lru_order, int64_t slot_count,
                        int64_t free_target, const int32_t* block_table, int64_t block_table_len, const void* kv0_src,
                        const void* kv1_src, void* kv0_dst, void* kv1_dst, int64_t kv0_row_bytes,
                        int64_t kv1_row_bytes, int64_t src_rows, int64_t max_seq_len, int64_t actual_seq_len,
                        int64_t block_size, int32_t* resolved, int32_t* evicted, int32_t* evicted_count,
                        int64_t* stats, int32_t* status);

/* asu_resolver_reset for `layers` layers in one launch: token_state / asu_record_addr /
 * hbm_slot_of_token are [layers, max_seq_len], slot_owner_token / free_slot_stack are
 * [layers, slot_count] and free_slot_count is [layers], all contiguous; every layer gets the same
 * reset (one request, one block table).  The reference resets layer by layer (patch/0003
 * ASUFullKVCacheManagerFunctional.reset_single_request, patch lines 411-426). */
int asu_resolver_reset_layers(void* stream, int64_t layers, int32_t* token_state, int32_t* asu_record_addr,
                              int32_t* hbm_slot_of_token, int64_t max_seq_len, int32_t* slot_owner_token,
                              int32_t* free_slot_stack, int32_t* free_slot_count, int64_t slot_count,
                              const int32_t* block_table, int64_t block_table_len, int64_t block_size,
                              int64_t actual_seq_len, int64_t managed_prefix_len);

/* Replaces ASUFullKVCacheManagerFunctional.mark_decode_token (patch/0003, patch lines 294-298 and
 * 428-432: token_state[token_id] = TAIL_HBM in every layer) with one launch over a
 * [layers, max_seq_len] token_state.  Rejects token_id outside [0, max_seq_len). */
int asu_resolver_mark_token(void* stream, int64_t layers, int32_t* token_state, int64_t max_seq_len,
                            int64_t token_id);

/* No counterpart in the reference.  The same resolver as asu_kv_resolver_do, for callers that
 * cannot allocate device memory while resolving (an engine whose HBM is pre-reserved for its
 * KV-block pool and that forbids cudaMalloc in the decode loop; a C / FFI host without a
 * caching allocator): the install-list scratch is a fixed device array inside the library,
 * ASU_RESOLVER_NOALLOC_MAX_TOPK entries (128 KiB per GPU that loads the library, held until
 * exit).  Larger topk_numel returns ASU_ERR_NOALLOC_CAPACITY and launches nothing.  The first
 * call on a device looks up the array's device address; make it before any stream capture.
 * All calls on a device share the array: calls whose launches overlap on the GPU race, so
 * order them on one stream.  Allocates nothing (no cudaMalloc / cudaFree). */
#define ASU_RESOLVER_NOALLOC_MAX_TOPK 16384
#define ASU_ERR_NOALLOC_CAPACITY (-3) /* topk_numel above ASU_RESOLVER_NOALLOC_MAX_TOPK */
int asu_kv_resolver_noalloc(void* stream, const int32_t* topk, int64_t topk_numel, int32_t* token_state,
                            const int32_t* asu_record_addr, int32_t* hbm_slot_of_token, int32_t* slot_owner_token,
                            const int32_t* free_slot_stack, int32_t* free_slot_count, int64_t free_slot_stack_len,
                            const int32_t* block_table, int64_t block_table_len, const void* kv0_src,
                            const void* kv1_src, void* kv0_dst, void* kv1_dst, int64_t kv0_row_bytes,
                            int64_t kv1_row_bytes, int64_t src_rows, int64_t slot_count, int64_t max_seq_len,
                            int64_t actual_seq_len, int64_t block_size, int32_t* resolved, int32_t* status);

#ifdef __cplusplus
}
#endif

#endif /* ASU_B200_H */
