/*
 * slotstream_b200.h -- C ABI of the B200-native (sm_100a) MoE hot path of slotstream-spark.
 *
 * Every entry point takes raw device pointers, element counts and a cudaStream_t passed as void*; none
 * allocates device memory, none synchronises the host, and every launch goes to the given stream, so
 * the calls can be captured in a CUDA graph -- except the ssb_pool_* calls of the slot pool, which own
 * device memory (create / resize allocate it, destroy synchronises) and are host-side. Each returns SSB_OK (0), a negative SSB_E* code for a bad
 * argument (checked before any launch), or a positive cudaError_t from the launch.
 *
 * Conventions: bf16 tensors are passed as uint16_t* bit patterns; 4-bit affine weights follow MLX
 * (element i of a row in bits [4*(i%8), 4*(i%8)+4) of int32 word i/8, w = q*s + b with bf16 s, b per
 * group of gs elements). An expert record is the reference's nine-piece layout (gate/up/down x w/s/b)
 * with offsets derived from (hidden, inter, gs).
 *
 * "Replaces" names the reference interface (file:line inside fortil/slotstream-spark) whose Python
 * function dispatches to the entry point in this build.
 */
#ifndef SLOTSTREAM_B200_H
#define SLOTSTREAM_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes */
#define SSB_OK 0
#define SSB_EINVAL (-1)       /* null pointer, count or size out of range */
#define SSB_EUNSUPPORTED (-2) /* a shape these kernels do not handle (see each entry point) */
#define SSB_ENODEVICE (-3)    /* current device is not sm_100 */
#define SSB_ETOOBIG (-4)      /* request larger than a fixed capacity (static scratch, slot pool) */
#define SSB_ETIMEDOUT (-5)    /* a bounded host-side wait gave up (ssb_wait_seq) */

/* ---- bits of the device error word (int32, caller-owned, OR-ed by kernels; never cleared by them) */
#define SSB_ERR_EXPERT_RANGE 1 /* an expert id outside [0, 512) */
#define SSB_ERR_UNMAPPED 2     /* map[layer*512 + e] < 0: the expert is not in the pool */
#define SSB_ERR_SLOT_RANGE 4   /* a slot index outside slot_ptr */
#define SSB_ERR_MISALIGNED 8   /* a record base that is not 16-byte aligned */
#define SSB_ERR_TIMEOUT 16     /* a bounded device-side wait gave up (the kernel skipped its work) */

/* ---- dtype tags for activations */
#define SSB_BF16 0
#define SSB_F32 1

/* Library version string. */
const char* ssb_version(void);

/* SSB_OK when the current device is an sm_100 part (B200), SSB_ENODEVICE otherwise. */
int ssb_device_check(void);

/* Static + dynamic shared memory (bytes) that the named kernel family last launched with; -1 if the
 * name is unknown or the kernel has not launched. Backs the reference's SHARED_BYTES bookkeeping
 * (slotstream_spark/kernels/gemv_affine.py:15-25). */
int ssb_kernel_smem(const char* name);

/* Number of SMs the persistent grouped GEMMs (ssb_prefill_experts, ssb_fused_moe_*, ssb_gemm_dense) leave
 * free at their next launches (default 0: one CTA on every SM), so that kernels on another stream -- the
 * all-to-all of an expert-parallel exchange -- can run beside them. A process-wide setting read at each launch.
 * No counterpart in the reference (it runs on one GPU with no collective to overlap). */
int ssb_set_gemm_sm_reserve(int32_t sms);

/* B-rows per tile of the sorted gate_up GEMM (ssb_sorted_gate_up, ssb_prefill_experts): 256 (default: 128 gate +
 * 128 up rows, M128 x N256 tensor-core instructions, one accumulator set that the epilogue hands back half by half)
 * or 128 (64 + 64 rows, M128 x N128 instructions, double-buffered accumulators). Both give the same bits. A
 * process-wide setting read at each launch; SSB_EINVAL for other values. No counterpart in the reference (a
 * Triton autotuning choice there, kernels/tuning.py). */
int ssb_set_gate_up_tile(int32_t b_rows);

/* Bound, in nanoseconds, of the grid-barrier waits of the cooperative kernels (ssb_moe_decode_fused; default 250 ms):
 * a barrier that does not complete in time gives up, the kernel sets SSB_ERR_TIMEOUT in the caller's error word
 * and returns (its outputs are then not valid, and its sync word must be zeroed before the next call). A
 * process-wide setting read at each launch; waits on the kernels' own copies keep their fixed bound. No
 * counterpart in the reference (its kernels do not wait on one another). */
int ssb_set_wait_limit_ns(int64_t ns);

/* Stable top-k of each row of fp32 scores [rows, n] (n <= 65536, 1 <= k <= n): order-preserving uint32
 * keys (NaN lowest), ties to the lower index; k <= 16 sorted by (value desc, index asc), larger k by
 * index asc; rows with fewer than k valid entries pad with index -1 / value -inf. n_valid (int32 [rows])
 * and out_val may be NULL.
 * Replaces: slotstream_spark/kernels/topk_stable.py:85-113 (kernel :28-82). */
int ssb_topk_stable(const float* scores, const int32_t* n_valid, int64_t rows, int32_t n, int32_t k,
                    int32_t* out_idx, float* out_val, void* stream);

/* Router logits: logits[t, j] = sum_h x[t, h] * w[j, h] for j < n_rows, fp32 accumulation of the exact
 * bf16 products; when w_extra != NULL one more column (index n_rows) is sum_h x[t, h] * w_extra[h].
 * x bf16 [tokens, hidden], w bf16 [n_rows, hidden] row-major, logits fp32 [tokens, ld]
 * (ld >= n_rows + (w_extra != NULL)). hidden must be a multiple of 256 and <= 4096.
 * Replaces: the router GEMV of model/layers.py:339 (lin -> kernels/gemv_affine.py:177-198). */
int ssb_router_logits(const uint16_t* x, const uint16_t* w, const uint16_t* w_extra, int64_t tokens,
                      int32_t hidden, int32_t n_rows, int32_t ld, float* logits, void* stream);

/* Router selection, one warp per token: (optional bf16 rounding of the logits), + bias[e] (optional,
 * fp32 [experts]), fp32 softmax over `experts` columns, stable top-k on the probabilities (same key rule
 * as ssb_topk_stable), renormalised weights w = p / sum(p). experts <= 1024, k <= 32.
 * out_probs (fp32 [tokens, experts]) may be NULL. With SSB_ROUTER_SHARED_GATE, column `experts` of the
 * logits is the shared-expert gate logit and out_sh_gate[t] = sigmoid(it).
 * Replaces: model/layers.py:340-347 (softmax, topk_stable, renormalise) and the shared-expert gate of
 * model/layers.py:401. */
#define SSB_ROUTER_ROUND_BF16 1
#define SSB_ROUTER_SHARED_GATE 2
int ssb_router_select(const float* logits, int32_t ld, int64_t tokens, int32_t experts, int32_t k,
                      const float* bias, int32_t flags, int32_t* out_idx, float* out_w, float* out_probs,
                      float* out_sh_gate, void* stream);

/* Stable counting sort of rows by local expert, padded per expert to block_m with the sentinel `rows`.
 * local = expert_map ? expert_map[row_expert[i]] (-1 when row_expert[i] is outside [0, map_len))
 *                    : row_expert[i];
 * rows with local outside [0, num_local) are dropped. Outputs: sorted_rows int32 [P], block_expert int32
 * [P / block_m] (-1 past num_padded), num_padded int32 [1], P = padded_rows(rows, num_local, block_m).
 * num_local <= 1280.
 * Replaces: slotstream_spark/kernels/moe_align.py:17-48 and align_rows of
 * slotstream_spark/kernels/fused_moe_affine.py:130-133. */
int ssb_moe_align(const int32_t* row_expert, int64_t rows, const int32_t* expert_map, int32_t map_len,
                  int32_t num_local, int32_t block_m, int32_t* sorted_rows, int32_t* block_expert,
                  int32_t* num_padded, void* stream);

/* Decode grouped GEMV over routed experts found through the slot tables:
 *   base(r, j) = slot_ptr[map[layer*512 + ids[r, j]]]
 *   h[r, j, :] = silu(G x_r) * (U x_r)                  (fp32, exact fp32 dequant algebra)
 *   o[r, j, :] = w[r, j] * (D h[r, j, :])               (fp32)
 *   out[r, :]  = o[r, 0] + o[r, 1] + ... in rank order  (sequential fp32)
 * x bf16|fp32 [rows, hidden] (x_dtype SSB_BF16 / SSB_F32); h_buf fp32 [rows, topk, inter];
 * o_buf fp32 [rows, topk, hidden] (nullable); out fp32 [rows, hidden]. hidden % 512 == 0 and <= 4096,
 * inter % 64 == 0 and <= 2048 (other shapes: SSB_EUNSUPPORTED), gs 64. With o_buf and rows >= 3 (rows * topk
 * <= 1024) the (row, rank) entries are grouped by expert, so a record chosen by several rows is read once;
 * the results are the same bits either way. err (int32, nullable) gets SSB_ERR_* bits; a bad expert
 * contributes zero. Row-invariant and placement-invariant bit for bit.
 * Replaces: slotstream_spark/kernels/moe_gemv_affine.py:113-147 (kernels :55-110). */
int ssb_moe_decode(const void* x, int32_t x_dtype, const int32_t* expert_ids, const float* weights,
                   int64_t rows, int32_t topk, int32_t hidden, int32_t inter, int32_t layer,
                   const int32_t* map_t, int64_t map_len, const int64_t* slot_ptr_t, int64_t n_slots,
                   float* h_buf, float* o_buf, float* out, int32_t* err, void* stream);

/* Fused decode layer (additive): ssb_moe_decode plus the shared expert, whose record sits at
 * shared_record, gated by sh_gate[r] (the sigmoid from ssb_router_select):
 *   sh[r, :] = sh_gate[r] * (D_s (silu(G_s x_r) * (U_s x_r)))
 *   y[r, :]  = bf16( bf16(out[r, :]) + bf16(sh[r, :]) )      (bf16 [rows, hidden])
 * h_buf must hold rows * (topk + 1) * inter floats (the shared expert's h follows the routed ones).
 * expert_base (nullable) holds the resolved record base of every (row, rank) from ssb_router_select_resolve.
 * flags bit 0 (SSB_DECODE_PDL): launch with programmatic dependent launch.
 * Replaces: the decode MoE call site of slotstream_spark/runtime/graphs.py:160-169 (moe_decode + shared
 * expert + routed.to(bf16) + sh). */
#define SSB_DECODE_PDL 1
int ssb_moe_decode_layer(const uint16_t* x, const int32_t* expert_ids, const float* weights, int64_t rows,
                         int32_t topk, int32_t hidden, int32_t inter, int32_t layer, const int32_t* map_t,
                         int64_t map_len, const int64_t* slot_ptr_t, int64_t n_slots, const void* shared_record,
                         const float* sh_gate, const int64_t* expert_base, float* h_buf, float* o_buf, float* out,
                         uint16_t* y, int32_t flags, int32_t* err, void* stream);

/* ssb_router_select plus expert resolution for the decode layer (additive): for every chosen expert the
 * record base slot_ptr[map[layer*512 + e]] is written to out_base [tokens, k] (0 when unmapped; SSB_ERR_* bits
 * in err) and the first prefetch_bytes of the record are prefetched into L2, so the expert GEMVs that follow
 * read resolved addresses from a warm cache. Pass out_base as ssb_moe_decode_layer's expert_base.
 * Replaces: the slot lookup of slotstream_spark/kernels/moe_gemv_affine.py:66-69 ahead of the GEMVs. */
int ssb_router_select_resolve(const float* logits, int32_t ld, int64_t tokens, int32_t experts, int32_t k,
                              const float* bias, int32_t flags, int32_t* out_idx, float* out_w, float* out_sh_gate,
                              int32_t layer, const int32_t* map_t, int64_t map_len, const int64_t* slot_ptr_t,
                              int64_t n_slots, int64_t* out_base, int64_t prefetch_bytes, int32_t* err, void* stream);

/* ---- expert-parallel prefill (experts sharded over n_ranks <= 8 GPUs; the exchange itself is NCCL
 * all-to-all-v between these calls). Placement: strided = 1 puts expert e on rank e % n_ranks (local index
 * e / n_ranks), strided = 0 on rank e / experts_per_rank (local e % experts_per_rank). k <= 15.
 * Replaces: no counterpart in the reference, which runs on one GPU; the per-rank expert work is
 * ssb_prefill_experts and the sums keep the rank order of kernels/fused_moe_affine.py:164-172. */

/* Dispatch plan of one rank's routed tokens ids/w [tokens, k]: dest_count int32 [n_ranks, 2] (rows, entries
 * per destination); send_token int32 [>= tokens * min(n_ranks, k)] (rows ordered by destination, then
 * token); send_meta int32 [same, 2k + 2] (local expert or -1 per choice, weight bits, entry base, entry
 * count); tok_slot / tok_entry int32 [tokens, n_ranks] (send row and entry base of (t, d), -1 if none).
 * tokens = 0 only zeroes dest_count (the other pointers may be NULL). */
int ssb_ep_plan(const int32_t* ids, const float* w, int64_t tokens, int32_t k, int32_t experts_per_rank,
                int32_t n_ranks, int32_t strided, int32_t* dest_count, int32_t* send_token, int32_t* send_meta,
                int32_t* tok_slot, int32_t* tok_entry, int32_t* err, void* stream);

/* dst[i] = src[idx[i]] for rows of row_bytes (multiple of 16) bytes; an index outside [0, src_rows) gives a
 * zero row and SSB_ERR_EXPERT_RANGE in err. */
int ssb_gather_rows(const void* src, int64_t src_rows, const int32_t* idx, int64_t n, int64_t row_bytes, void* dst,
                    int32_t* err, void* stream);

/* Received metadata [rows, 2k + 2] (rows of source s at src_row_off[s] .. src_row_off[s+1], their entries at
 * src_entry_off[s] ..) -> compacted entries row_expert / row_token / row_weight [n_entries] (entries of a row
 * contiguous in rank-k order) and row_e0 int64 / row_cnt int32 [rows]. */
int ssb_ep_unpack(const int32_t* meta, int64_t rows, int32_t k, const int32_t* src_row_off,
                  const int64_t* src_entry_off, int32_t n_ranks, int64_t n_entries, int32_t* row_expert,
                  int32_t* row_token, float* row_weight, int64_t* row_e0, int32_t* row_cnt, int32_t* err,
                  void* stream);

/* partial[r, :] = rows[row_e0[r]] + ... + rows[row_e0[r] + row_cnt[r] - 1], sequential fp32. */
int ssb_combine_rows(const float* rows, const int64_t* row_e0, const int32_t* row_cnt, int64_t n, int32_t hidden,
                     float* partial, void* stream);

/* The same sums rounded to bf16 (round to nearest even): a half-size partial-sum return for the exchange. */
int ssb_combine_rows_bf16(const float* rows, const int64_t* row_e0, const int32_t* row_cnt, int64_t n,
                          int32_t hidden, uint16_t* partial, void* stream);

/* Home combine of the returned rows: exact = 0 sums the partial rows ret[tok_slot[t, d]] over d ascending;
 * exact = 1 sums the entry rows ret[ret_entry_off[d] + tok_entry[t, d] + i] in router-rank order (bit-equal
 * to the one-GPU layer). out fp32 [tokens, hidden] (nullable); y bf16 = bf16(bf16(routed) + bf16(sh))
 * (nullable; sh fp32 bf16-valued [tokens, hidden], nullable). */
int ssb_ep_combine(const float* ret, const int32_t* tok_slot, const int32_t* tok_entry, const int64_t* ret_entry_off,
                   const int32_t* ids, int64_t tokens, int32_t k, int32_t experts_per_rank, int32_t n_ranks,
                   int32_t strided, int32_t exact, int32_t hidden, const float* sh, float* out, uint16_t* y,
                   void* stream);

/* Home combine of bf16 partial rows (ssb_combine_rows_bf16 on the destinations): routed[t] = sum over d ascending
 * of float(ret[tok_slot[t, d]]) in fp32; out / y as ssb_ep_combine. */
int ssb_ep_combine_bf16(const uint16_t* ret, const int32_t* tok_slot, const int32_t* ids, int64_t tokens, int32_t k,
                        int32_t experts_per_rank, int32_t n_ranks, int32_t strided, int32_t hidden, const float* sh,
                        float* out, uint16_t* y, void* stream);

/* ---- HBM expert slot pool for streaming decode (additive; the B200 side of slotio's Pool + Ensurer,
 * slotio/include/slotio/pool.hpp:23-160 and slotio/src/ensure.cpp). Unlike the kernel entry points, the pool
 * owns device memory: ssb_pool_create allocates the device tables map (int32 [layers * experts], -1 = absent)
 * and slot_ptr (int64 [max_slots]) on the current device, ssb_pool_resize the 1 GiB chunks that hold the slots.
 * The decode entry points read experts through these two tables (ssb_pool_tables). Not thread-safe across
 * pools; calls on one pool are serialised by its lock. */
typedef struct ssb_pool ssb_pool;
ssb_pool* ssb_pool_create(int64_t record_bytes, int64_t chunk_bytes, int32_t layers, int32_t experts,
                          int32_t max_slots);
void ssb_pool_destroy(ssb_pool* pool);
/* Grow to n_slots slots (allocating whole chunks); shrinking is not supported. */
int ssb_pool_resize(ssb_pool* pool, int32_t n_slots);
int ssb_pool_tables(ssb_pool* pool, int32_t** map_dev, int64_t** slot_ptr_dev, int64_t* map_len, int32_t* n_slots,
                    int32_t* chunks);
/* Make experts[0..n) of `layer` resident before the layer's kernels run on compute_stream. Duplicates are
 * allowed; hits are marked referenced; each miss takes a CLOCK victim (never a slot this call needs), is copied
 * from host_table[layer * experts + e] (pinned host record) on copy_stream after the victim's last reader
 * (see ssb_pool_release) has finished, and is published in map on copy_stream; compute_stream then waits for
 * the copies (either stream may be 0, the default stream). out_slots[i] (host, nullable) = slot of experts[i];
 * stats (host int64 [3], nullable) = hits,
 * misses, bytes copied by this call. SSB_ETOOBIG when the misses do not fit (nothing changed).
 * Replaces: Ensurer::ensure, slotio/include/slotio/pool.hpp:141-160 (slotio/src/ensure.cpp). */
int ssb_pool_ensure(ssb_pool* pool, int32_t layer, const int32_t* experts, int32_t n, const void* const* host_table,
                    void* copy_stream, void* compute_stream, int32_t* out_slots, int64_t* stats);
/* Record, on compute_stream after the kernels of the last ensured layer, the event that every slot that
 * layer used waits for before it can be overwritten. */
int ssb_pool_release(ssb_pool* pool, void* compute_stream);
int ssb_pool_counters(ssb_pool* pool, int64_t* hits, int64_t* misses, int64_t* bytes);

/* One decode MoE layer streaming its experts through the pool (host-side; it waits for the router): router
 * logits and select with the shared gate (as ssb_router_logits + ssb_router_select: logits_ws fp32
 * [rows, experts + 1], ids int32 / w fp32 [rows, topk], sh_gate fp32 [rows]), the ids copied to ids_host
 * (pinned int32 [rows, topk]), ssb_pool_ensure for them (stats as there), ssb_moe_decode_layer through the
 * pool's tables on compute_stream (h_buf, o_buf, out, y, err as there), then ssb_pool_release.
 * Replaces: the per-layer sequence of slotstream_spark/model/layers.py:372-385 (seg_moe: router ids to the host,
 * pool.ensure, the MoE kernels through the pool's tables) and runtime/graphs.py:316-323. */
int ssb_pool_decode_layer(ssb_pool* pool, int32_t layer, const uint16_t* x, int64_t rows, int32_t topk,
                          int32_t hidden, int32_t inter, int32_t experts, const uint16_t* w_router,
                          const uint16_t* sh_gate_w, const float* bias, const void* const* host_table,
                          const void* shared_record, float* logits_ws, int32_t* ids, float* w, float* sh_gate,
                          int32_t* ids_host, float* h_buf, float* o_buf, float* out, uint16_t* y, int32_t* err,
                          void* copy_stream, void* compute_stream, int64_t* stats);

/* Host-side helper: one asynchronous copy of `bytes` bytes (cudaMemcpyAsync, direction from the addresses) on
 * `stream`, for callers that hold raw record addresses -- the prefill sweep stages non-resident records from pinned
 * host memory with it. Replaces: the staging reads of slotio's Sweep (slotstream_spark/model/moe_sweep.py:113-121)
 * for records already in pinned host memory. */
int ssb_copy_async(void* dst, const void* src, int64_t bytes, void* stream);

/* Router logits + select (as ssb_router_logits then ssb_router_select) with the logits held in a fixed
 * device array that comes with the library's device code, so the call needs no workspace and allocates nothing:
 * for callers that cannot allocate on their call path (a host binding without a caching allocator, which would
 * need a device-synchronising cudaMalloc per step; a process whose slot pool holds nearly all HBM). Capacity: 65536 floats
 * (256 KiB); tokens * (experts + 1 when w_shared_gate is given, else experts) above it returns SSB_ETOOBIG
 * before any launch. flags: 0 or SSB_ROUTER_ROUND_BF16; a non-null w_shared_gate (bf16 [hidden]) adds the
 * shared gate into out_sh_gate. The array is shared by every call on a device: calls that overlap on one
 * device (other streams or host threads) race. The first call on each device looks up the array's address and
 * keeps it for the life of the process: make that first call before any stream capture, and do not reset the
 * device (cudaDeviceReset) while the library is loaded. Other limits as ssb_router_logits and ssb_router_select.
 * Replaces: no counterpart in the reference. */
int ssb_router_topk_static(const uint16_t* x, const uint16_t* w, const uint16_t* w_shared_gate, int64_t tokens,
                           int32_t hidden, int32_t experts, int32_t k, const float* bias, int32_t flags,
                           int32_t* out_idx, float* out_w, float* out_sh_gate, void* stream);

/* Whole decode MoE layer for rows <= 2 tokens in ONE cooperative launch (one CTA per SM, two grid barriers):
 * router logits (x . w_router^T and the shared gate x . sh_gate_w, fp32), select as ssb_router_select (bias,
 * flags SSB_ROUTER_ROUND_BF16), expert resolution through the slot tables as ssb_moe_decode, then gate_up / down /
 * rank-order sum / shared add. Two kernels: on CUDA cores (exact fp32 dequantisation algebra; h, out and y equal
 * ssb_moe_decode_layer's bit for bit), and on the tensor cores (4-bit codes dequantised exactly to bf16, fp32
 * accumulation, the affine scale and bias applied per 64-element group in fp32, h kept in fp32 as a bf16 hi + lo
 * pair; each distinct chosen expert read once for both tokens; h, out and y within the exact path's tolerance,
 * relative L2 1e-4). Both give out_idx / out_w / out_sh_gate / out_base equal to the separate calls bit for bit.
 * flags SSB_DECODE_FUSED_CUDA_CORES / SSB_DECODE_FUSED_TENSOR_CORES pick one; by default one token runs on CUDA
 * cores and two on the tensor cores (the faster of the two for each, measured on B200). The tensor-core kernel
 * falls back to the CUDA-core one for a shape it does not take (hidden other than 2048 / 2560 / 4096, inter not a
 * multiple of 128, or more resident weight rows per SM than its shared memory holds). Outputs: out_idx / out_w [rows, topk], out_sh_gate [rows], out_base
 * [rows, topk] (nullable), h_buf [rows * (topk + 1), inter] (16-byte aligned), o_buf [rows, topk, hidden]
 * (nullable), out fp32 / y bf16 [rows, hidden]. logits_ws: fp32 [rows, experts + 1]. sync: two uint32 words,
 * zero before the first call and after a call that reported SSB_ERR_TIMEOUT; calls sharing sync must not overlap.
 * Limits: hidden % 512 == 0 and <= 4096, inter in {512, 1024, 2048} (tensor cores: any multiple of 128 up to
 * 2048), experts <= 512, topk <= 16, gs 64; other shapes return SSB_EUNSUPPORTED.
 * Replaces: the router of model/layers.py:336-347 plus the decode MoE call site of
 * slotstream_spark/runtime/graphs.py:160-169, for callers that opt in. */
#define SSB_DECODE_FUSED_CUDA_CORES 4
#define SSB_DECODE_FUSED_TENSOR_CORES 8
int ssb_moe_decode_fused(const uint16_t* x, int64_t rows, int32_t topk, int32_t hidden, int32_t inter, int32_t experts,
                         const uint16_t* w_router, const uint16_t* sh_gate_w, const float* bias, int32_t flags,
                         int32_t layer, const int32_t* map_t, int64_t map_len, const int64_t* slot_ptr_t,
                         int64_t n_slots, const void* shared_record, float* logits_ws, int32_t* out_idx, float* out_w,
                         float* out_sh_gate, int64_t* out_base, float* h_buf, float* o_buf, float* out, uint16_t* y,
                         uint32_t* sync, int32_t* err, void* stream);

/* Router readback signal (one warp, graph-capturable): copies ids int32 / w fp32 [n] (n <= 32; n = 0 publishes only)
 * into slot `layer` of slot_ids / slot_w (32 elements per layer; pinned host buffers the device writes through their
 * mapping), then publishes *seq = ctrl[1] + layer with a system-scope release exchange, so a host thread that observes
 * seq >= ctrl[1] + layer with an acquire load (ssb_wait_seq) also sees that layer's ids and weights. ctrl int64 [2]
 * (position, step base) is written by the host before the step's graph launches.
 * Replaces: signal(), slotstream_spark/kernels/signal.py:15-37 (kernel :15-26). */
int ssb_signal(const int32_t* ids, const float* w, int32_t n, int32_t* slot_ids, float* slot_w, int64_t* seq,
               const int64_t* ctrl, int32_t layer, void* stream);

/* Host-side: spin (acquire loads, yielding every 256 polls) until *seq >= target; SSB_ETIMEDOUT after timeout_ns.
 * Replaces: Readback.wait / slotio.wait_seq, slotstream_spark/runtime/readback.py:40-46. */
int ssb_wait_seq(const int64_t* seq, int64_t target, int64_t timeout_ns);

/* Copy `bytes` (at most 16 MiB) with the SMs' own loads and stores on `stream`, between device memory and pinned
 * host memory (which the GPU addresses directly) or within either. For the small host reads and writes of a
 * step (counts, offsets) that must not queue on a copy engine behind a large transfer of another stream -- the
 * previous step's output leaving, the next step's input arriving. Pinned host memory must stay allocated until
 * the copy has run (a wait on `stream`). No counterpart in the reference (its host reads are synchronous). */
int ssb_copy_sm(void* dst, const void* src, int64_t bytes, void* stream);

/* Hint: bring [p, p + bytes) of device memory into L2 on `stream` (bulk L2 prefetches; nothing is written). A
 * decode step can issue it on a side stream for the next layer's router weight and shared-expert record, which
 * do not depend on routing, while the current layer streams its experts (opt-in: measured slower in the
 * 48-layer graph). No counterpart in the reference. */
int ssb_prefetch_l2(const void* p, int64_t bytes, void* stream);

/* Rank-order combine: out[t, :] = rows[t*k] + rows[t*k + 1] + ... sequentially in fp32.
 * rows fp32 [tokens * k, hidden], out fp32 [tokens, hidden]; hidden % 4 == 0.
 * Replaces: combine_rank_order, slotstream_spark/kernels/fused_moe_affine.py:164-172. */
int ssb_combine_rank_order(const float* rows, int64_t tokens, int32_t k, int32_t hidden, float* out,
                           void* stream);

/* Layer combine (additive): the rank-order sum above, then y[t, :] = bf16(bf16(sum) + bf16(sh[t, :]))
 * (sh fp32 [tokens, hidden], nullable = no shared expert); out (nullable) also receives the fp32 sum.
 * Replaces: the combine_rank_order + routed.to(bf16) + sh sequence of model/moe_sweep.py:161 and
 * engine/prefill.py:200-201. */
int ssb_combine_layer(const float* rows, int64_t tokens, int32_t k, int32_t hidden, const float* sh, float* out,
                      uint16_t* y, void* stream);

/* Prefill grouped GEMM, gate/up half, on tcgen05 tensor cores (M128 N128 K16 MMAs, fp32 in TMEM):
 *   h[row, :] = bf16( silu(x[row_token[row]] G_e^T) * (x[row_token[row]] U_e^T) )
 * for every row of every 256-row block b < num_padded/256 of the moe_align output (block_m = 256),
 * e = block_expert[b], record base group_ptr[e]. The dequantised tiles are rounded to bf16 (q*s + b in fp32
 * first) and accumulated in fp32, the reference's rounding path. x bf16 [tokens, hidden]; h_buf bf16
 * [rows, inter]; padded_len = sorted_rows length (a multiple of 256). hidden % 64 == 0 and (hidden/64) even,
 * inter % 64 == 0.
 * Replaces: launch_gate_up / _gate_up_kernel, slotstream_spark/kernels/fused_moe_affine.py:53-81, 111-118. */
int ssb_fused_moe_gate_up(const uint16_t* x, int64_t tokens, int32_t hidden, int32_t inter, const int32_t* row_token,
                          int64_t rows, const int32_t* sorted_rows, const int32_t* block_expert,
                          const int32_t* num_padded, int64_t padded_len, const int64_t* group_ptr, int32_t n_groups,
                          uint16_t* h_buf, int32_t* err, void* stream);

/* Prefill grouped GEMM, down half: out_rows[row, :] = (h[row] D_e^T) * row_weight[row], fp32; rows outside
 * the aligned blocks (block_m = 256) are left untouched. inter % 64 == 0 and (inter/64) even, hidden % 128 == 0.
 * Replaces: launch_down / _down_kernel, slotstream_spark/kernels/fused_moe_affine.py:84-108, 121-127. */
int ssb_fused_moe_down(const uint16_t* h_buf, int64_t rows, int32_t hidden, int32_t inter, const float* row_weight,
                       const int32_t* sorted_rows, const int32_t* block_expert, const int32_t* num_padded,
                       int64_t padded_len, const int64_t* group_ptr, int32_t n_groups, float* out_rows, int32_t* err,
                       void* stream);

/* Both prefill expert GEMMs of a fused MoE layer (additive), on activation rows permuted into expert order:
 * the rows of x copied into expert order (as ssb_permute_rows, but in row order through their sorted positions,
 * and without writing the padding rows, whose results no GEMM stores), then ssb_sorted_gate_up, then
 * ssb_sorted_down below, so the grouped GEMMs read whole 256-row 2-D tiles instead of gathering rows (align
 * with block_m = 256). Local expert `shared_local` (-1: none) is the shared expert --
 * its h is bf16(bf16(silu(bf16 g)) * bf16 u) and its down rows bf16(row_weight * bf16(h D^T)), the
 * reference's bf16 rounding between the shared expert's ops (model/moe_sweep.py:37-43) -- so it rides in the
 * same grouped launch as the routed experts with its rows weighted by the sigmoid gate. x holds `tokens` rows
 * (row_token < tokens); x_sorted bf16 [padded_len, hidden] and h_sorted bf16 [padded_len, inter] are scratch
 * (h in sorted order; h_sorted first holds the rows' sorted positions); out_rows fp32 [rows, hidden] indexed by
 * row as ssb_fused_moe_down.
 * Replaces: the per-group fused_moe_affine calls of model/moe_sweep.py:163-176 plus shared_expert
 * (:37-43) for a layer whose experts are all resident. */
int ssb_prefill_experts(const uint16_t* x, int64_t tokens, int32_t hidden, int32_t inter,
                        const int32_t* row_token, const float* row_weight, int64_t rows, const int32_t* sorted_rows,
                        const int32_t* block_expert, const int32_t* num_padded, int64_t padded_len,
                        const int64_t* group_ptr, int32_t n_groups, int32_t shared_local, uint16_t* x_sorted,
                        uint16_t* h_sorted, float* out_rows, int32_t* err, void* stream);

/* x_sorted[m, :] = x[row_token[sorted_rows[m]], :] for m < num_padded (zero rows for padding), with every group
 * of 8 columns in the K order (0,4,1,5,2,6,3,7): the order in which ssb_sorted_gate_up / ssb_sorted_down
 * dequantise their 4-bit weights (two codes per bf16x2 pair); h_sorted comes out in the same order. */
int ssb_permute_rows(const uint16_t* x, int64_t tokens, int32_t hidden, const int32_t* row_token, int64_t rows,
                     const int32_t* sorted_rows, const int32_t* num_padded, int64_t padded_len, uint16_t* x_sorted,
                     void* stream);

/* The gate_up GEMM of ssb_prefill_experts on permuted rows: h_sorted[m] = SwiGLU of x_sorted[m] for the
 * m-block's expert (shapes as ssb_fused_moe_gate_up). */
int ssb_sorted_gate_up(const uint16_t* x_sorted, int32_t hidden, int32_t inter, const int32_t* row_token,
                       int64_t rows, const int32_t* sorted_rows, const int32_t* block_expert, const int32_t* num_padded,
                       int64_t padded_len, const int64_t* group_ptr, int32_t n_groups, int32_t shared_local,
                       uint16_t* h_sorted, int32_t* err, void* stream);

/* The down GEMM of ssb_prefill_experts on h in sorted order: out_rows[sorted_rows[m]] = (h_sorted[m] D^T) * w. */
int ssb_sorted_down(const uint16_t* h_sorted, int64_t rows, int32_t hidden, int32_t inter, const float* row_weight,
                    const int32_t* sorted_rows, const int32_t* block_expert, const int32_t* num_padded,
                    int64_t padded_len, const int64_t* group_ptr, int32_t n_groups, int32_t shared_local,
                    float* out_rows, int32_t* err, void* stream);

/* Dense bf16 GEMM on tcgen05: out[m, n] = sum_k x[m, k] * w[n, k], fp32 into rows of `ldo` floats (ldo >= n).
 * k % 64 == 0, any n >= 1 (the last 128-column block is partial); row-invariant (fixed k order per output).
 * Replaces: gemm(x, DenseWeight), slotstream_spark/kernels/gemm_affine.py:40-59, 62-98 -- the dense lin() calls of
 * model/layers.py:62-76 inside prefill_gemm(), the router logits of a prefill chunk among them. */
int ssb_gemm_dense(const uint16_t* x, int64_t m, int32_t k, const uint16_t* w, int32_t n, float* out, int64_t ldo,
                   void* stream);

/* Dense prefill GEMM with an affine 4-bit weight on tcgen05: out[m, n] = sum_k x[m, k] * bf16(q*s + b)[n, k],
 * fp32 out [m, n]. k % 128 == 0, gs 32 or 64, any n >= 1; row-invariant (fixed k order per output).
 * Replaces: gemm(x, AffineWeight), slotstream_spark/kernels/gemm_affine.py:62-98 (kernel :19-37). */
int ssb_gemm_affine4(const uint16_t* x, int64_t m, int32_t k, const int32_t* q, const uint16_t* s, const uint16_t* b,
                     int32_t n, int32_t gs, float* out, void* stream);

/* Affine GEMV: out[r, i] = sum_j x[r, j] * (q[i, j] * s[i, j / gs] + b[i, j / gs]), fp32 accumulation,
 * bits 4 or 8, gs 32 or 64, k % 512 == 0 (4-bit) or k % 256 == 0 (8-bit), k <= 16384.
 * Row-invariant: each output row is the same op sequence whatever `rows` is.
 * Replaces: gemv(x, AffineWeight) of slotstream_spark/kernels/gemv_affine.py:214-262. */
int ssb_gemv_affine(const void* x, int32_t x_dtype, int64_t rows, const int32_t* q, const uint16_t* s,
                    const uint16_t* b, int32_t n, int32_t k, int32_t bits, int32_t gs, float* out, void* stream);

/* Dense bf16 GEMV: out[r, i] = sum_j x[r, j] * w[i, j], fp32 accumulation; k % 256 == 0, k <= 16384.
 * Replaces: gemv(x, DenseWeight) of slotstream_spark/kernels/gemv_affine.py:214-262. */
int ssb_gemv_dense(const void* x, int32_t x_dtype, int64_t rows, const uint16_t* w, int32_t n, int32_t k,
                   float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SLOTSTREAM_B200_H */
