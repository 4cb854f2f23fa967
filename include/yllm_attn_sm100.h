/* yllm_attn_sm100.h -- C ABI of the sm_100a (B200) attention path for the yllm engine.
 *
 * Plain pointers and sizes only.  Every q/k/v/out/state pointer is a DEVICE
 * pointer unless the comment says "host".  Streams are passed as void*
 * (a cudaStream_t; NULL = the legacy default stream the reference launches on).
 *
 * Two families of entry points:
 *   1. Drop-in replacements for the reference's CUDA launchers, same names and
 *      signatures as inference/cuda/cuda_kernels.h (void, legacy default
 *      stream).  A failure is kept in yattn_last_error() instead of silently
 *      launching nothing.
 *   2. yattn_* entry points that return 0 / -1 and fill (err, errlen), the
 *      cuda_k_gemv_f16 convention (inference/cuda/cuda_kernels.cu:53-87), and
 *      take an explicit stream and caller-owned workspace.
 *
 * KV cache layout (engine.c:261, 1066-1067; device_cuda.c:396-398): fp16 bits
 * (uint16_t), one region per layer, row t of a layer at base + t*kv_dim, the
 * kv_head slice at + kv_head*head_dim.  q and out are fp32, heads contiguous.
 * Query head hh reads kv head hh*n_kv_heads/n_heads (engine.c:1079).
 */
#ifndef YLLM_ATTN_SM100_H
#define YLLM_ATTN_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */

/* Library version (major*10000 + minor*100 + patch). */
int yattn_version(void);

/* Message of the last failure of a void drop-in entry point on this host
 * thread ("" if none).  Replaces the reference's silent early return
 * (cuda_kernels.cu:594, 651). */
const char* yattn_last_error(void);

/* Clears yattn_last_error() for this host thread. */
void yattn_clear_error(void);

/* Reads (and with clear != 0 resets) the device-side status word of the
 * current device: 0 = no kernel gave up; otherwise the code of the first
 * bounded wait that timed out (a kernel that times out returns early instead
 * of hanging), 103 if a decode run met a malformed work item (q or gate
 * not 16-byte aligned; with a pool, K/V not at a row of the pool) and
 * stopped, or 202 if a prefill told YATTN_PREFILL_Q_F16 met a q value that is
 * not an fp16 value.  It covers the allocation-free decode too, whose word sits in its
 * static scratch; polling creates neither word.  Synchronises the legacy
 * default stream. */
int yattn_device_status(int* status_out, int clear, char* err, size_t errlen);

/* ------------------------------------------------ drop-in replacements
 * Same names and signatures as the reference's inference/cuda/cuda_kernels.h. */

/* Replaces cuda_k_attn_decode (cuda_kernels.h:55-58; kernel cuda_kernels.cu:543-600).
 * One query token at position pos attends to keys 0..pos of one layer.
 * Split-KV over the sequence with a log-sum-exp merge; the split partials live
 * in a per-device workspace that the first call (or yattn_reserve) allocates. */
void cuda_k_attn_decode(float* att_out,
                        const float* q, const uint16_t* kcache, const uint16_t* vcache,
                        uint32_t pos, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                        uint32_t kv_dim);

/* Replaces cuda_k_attn_prefill (cuda_kernels.h:60-63; kernel cuda_kernels.cu:602-655).
 * B query tokens at positions pos_start..pos_start+B-1 (q row b at
 * q + b*q_stride); token b attends keys 0..pos_start+b.  Any B (the reference
 * caps a chunk at 64).  Flash attention on tcgen05 tensor cores with fp32
 * accumulation.  q (the engine's fp32 projections) is split into fp16 hi + lo
 * planes, about 22 significant bits, and both are multiplied into the scores;
 * |q| must stay below 65504.  P is split the same way.  Needs 16-byte aligned
 * pointers, q_stride % 4 == 0, kv_dim % 8 == 0, head_dim 64/128/256. */
void cuda_k_attn_prefill(float* att_out,
                         const float* q, const uint16_t* kcache, const uint16_t* vcache,
                         uint32_t pos_start, uint32_t B, uint32_t n_heads, uint32_t n_kv_heads,
                         uint32_t head_dim, uint32_t kv_dim, uint32_t q_stride);

/* Replaces cuda_k_store_kv (cuda_kernels.h:50-51; kernel cuda_kernels.cu:494-507).
 * Unlike the reference kernel (__float2half_rn, round-to-nearest-even) this
 * rounds with the engine's own f32_to_f16 (platform.c:340-379: half-up, f32
 * subnormals to zero), so the device cache bytes equal the CPU engine's. */
void cuda_k_store_kv(uint16_t* kcache, uint16_t* vcache, const float* k, const float* v,
                     uint32_t pos, uint32_t kv_dim);

/* Replaces cuda_k_store_kv_batch (cuda_kernels.h:52-53; cuda_kernels.cu:509-528), same rounding. */
void cuda_k_store_kv_batch(uint16_t* kcache, uint16_t* vcache, const float* k, const float* v,
                           uint32_t pos_start, uint32_t B, uint32_t kv_dim);

/* -------------------------------------------- fused RoPE + KV store (decode) */

/* One sequence's inputs of a decode step at one layer: q [n_heads*head_dim]
 * fp32 (rotated in place), k and v [n_kv_heads*head_dim] fp32 (read only),
 * the layer's K and V cache bases (row t at + t*kv_dim) and the position. */
typedef struct YattnRopeItem {
    float* q;
    const float* k;
    const float* v;
    uint16_t* kcache;
    uint16_t* vcache;
    uint32_t pos;
    uint32_t reserved;
} YattnRopeItem;

/* Optional QK-norm ahead of the rotation (qwen3: engine.c:1036-1045; qwen35:
 * engine.c:915-919): every q head and every k head becomes rmsnorm(x, w)
 * (matvec.c:152-165: y = x * w / sqrt(mean(x^2) + eps)) with the layer's
 * shared head_dim weights q_w / k_w (device pointers; fp32, or fp16 bits when
 * w_f16 != 0).  Passed by host pointer; NULL = no norm.  head_dim <= 256. */
typedef struct YattnQkNorm {
    const void* q_w;
    const void* k_w;
    int w_f16;
    float eps;
} YattnQkNorm;

/* RoPE of q and k at each item's position, then k (rotated) and v into the
 * cache at that position with the engine's f32_to_f16 rounding, for all
 * n_items (device array) in one launch.  Replaces, per sequence, the
 * reference's cuda_k_rope_{llama,qwen}_heads on q and on k plus
 * cuda_k_store_kv (cuda_fwd.c:136-147; CPU engine.c:1052-1072).
 * rope_kind: 0 = rope_inplace (pairs 2j, 2j+1; matvec.c:890-904),
 * 1 = rope_inplace_qwen (pairs j, j + head_dim/2; matvec.c:907-921),
 * 2 = rope_inplace_mrope (first n_rope_dims dims, pairs j, j + n_rope_dims/2;
 * matvec.c:924-939).  n_rope_dims is ignored for kinds 0 and 1.  The inverse
 * frequencies are the reference's powf values (computed on the host); the
 * device's sinf/cosf can move a stored fp16 value by one ulp.  With qk_norm,
 * q and k are first normalised per head (YattnQkNorm above; one CTA per head). */
int yattn_rope_store_kv(const YattnRopeItem* items_dev, uint32_t n_items, uint32_t n_heads,
                        uint32_t n_kv_heads, uint32_t head_dim, uint32_t kv_dim, int rope_kind,
                        uint32_t n_rope_dims, float theta, const YattnQkNorm* qk_norm, void* stream,
                        char* err, size_t errlen);

/* The same for B consecutive tokens of one sequence (a prefill chunk): row b
 * of q (at q + b*q_stride), k and v (at + b*kv_dim) is rotated at position
 * pos_start + b and stored into cache row pos_start + b.  Replaces the
 * batched cuda_k_rope_{llama,qwen}_heads_batch on q and k plus
 * cuda_k_store_kv_batch (cuda_fwd.c:207-218): one launch for the chunk. */
int yattn_rope_store_kv_batch(float* q, const float* k, const float* v, uint16_t* kcache,
                              uint16_t* vcache, uint32_t pos_start, uint32_t B, uint32_t q_stride,
                              uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, uint32_t kv_dim,
                              int rope_kind, uint32_t n_rope_dims, float theta,
                              const YattnQkNorm* qk_norm, void* stream, char* err, size_t errlen);

/* ---------------------------------------------- batched / split-KV decode */

/* One decode query: the attention of one sequence at one layer.
 * k, v: that layer's cache base (row t at k + t*kv_dim).  gate: NULL, or
 * [n_heads*head_dim] fp32 for the qwen35 output gate out *= sigmoid(gate)
 * (engine.c:958-960).  Keys 0..pos are attended. */
typedef struct YattnDecodeItem {
    const float* q;
    float* out;
    const uint16_t* k;
    const uint16_t* v;
    const float* gate;
    uint32_t pos;
    uint32_t reserved;
} YattnDecodeItem;

/* One CTA of work: keys [t_begin, t_end) of one item for a group of kv heads
 * (kv_head is the group's first head; a group is the largest of 8/4/2/1 heads
 * dividing n_kv_heads, at most 4 for head_dim 256, so one token's K row of the
 * group is one contiguous copy).  Filled by yattn_decode_plan; opaque to
 * callers apart from its size. */
typedef struct YattnDecodeWork {
    uint32_t item;
    uint16_t kv_head;
    uint16_t n_splits;
    uint32_t split;
    uint32_t t_begin;
    uint32_t t_end;
    uint32_t part_base;   /* first partial slot of this (item, head group); unused if n_splits == 1 */
    uint32_t group;       /* merge counter of this (item, head group); unused if n_splits == 1 */
    uint32_t cta;         /* CTA that streams this unit; units are grouped by cta, in order */
} YattnDecodeWork;

/* Host-side schedule.  pos_host[n_items] are the items' query positions.
 * split_tokens = 0: balanced plan.  The key ranges of every (item, head group)
 * are laid end to end and cut into target_ctas equal chunks (target_ctas = 0:
 * one per SM of the current device); a CTA streams its chunk as one or more
 * units (segments of one (item, head group) each), so every CTA moves the
 * same bytes.  split_tokens > 0: uniform splits of that length, one unit per
 * CTA, longest first.  Writes up to work_cap entries to work_host (host
 * memory).  The schedule depends only on the positions and the head geometry,
 * so one plan serves every layer of a decode step. */
int yattn_decode_plan(const uint32_t* pos_host, uint32_t n_items, uint32_t n_kv_heads,
                      uint32_t head_dim, uint32_t split_tokens, uint32_t target_ctas,
                      YattnDecodeWork* work_host, uint32_t work_cap,
                      uint32_t* n_work, uint32_t* n_parts, uint32_t* n_groups,
                      char* err, size_t errlen);

/* Workspace bytes for a plan (split partials + merge counters). */
size_t yattn_decode_workspace_bytes(uint32_t n_parts, uint32_t n_groups,
                                    uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim);

/* Zeroes the merge counters of a new workspace (runs leave them at zero). */
int yattn_decode_workspace_init(void* workspace, size_t ws_bytes, void* stream,
                                char* err, size_t errlen);

/* Runs a plan: items_dev[] and work_dev[] are device copies of the items and
 * of yattn_decode_plan's output.  Supported: head_dim 64/128/256, up to 8
 * query heads per kv head, kv_dim % 8 == 0, 16-byte aligned q, gate and k/v
 * bases.  Plans hold no empty key range (t_end > t_begin). */
int yattn_decode_run(const YattnDecodeItem* items_dev, const YattnDecodeWork* work_dev,
                     uint32_t n_work, uint32_t n_parts, uint32_t n_groups,
                     uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, uint32_t kv_dim,
                     void* workspace, size_t ws_bytes, void* stream, char* err, size_t errlen);

/* Pooled variants: every item's K and V rows lie in one allocation
 * [pool, pool + pool_bytes) with row stride kv_dim (the engine's per-sequence
 * blobs carved from one pool).  One 2-D tensor map covers the pool, so K and V
 * stream through tensor copies of 8-16 KB (64 dims x one stage of tokens,
 * 128-byte swizzle) instead of one copy per row -- the faster path.  A pooled
 * run needs a plan from yattn_decode_plan_pooled, which groups kv heads for
 * the tensor copies (two per CTA at head_dim <= 128 with an even n_kv_heads,
 * else one); the work array, workspace sizing and item layout are as above. */
int yattn_decode_plan_pooled(const uint32_t* pos_host, uint32_t n_items, uint32_t n_kv_heads,
                             uint32_t head_dim, uint32_t split_tokens, uint32_t target_ctas,
                             YattnDecodeWork* work_host, uint32_t work_cap,
                             uint32_t* n_work, uint32_t* n_parts, uint32_t* n_groups,
                             char* err, size_t errlen);
int yattn_decode_run_pooled(const YattnDecodeItem* items_dev, const YattnDecodeWork* work_dev,
                            uint32_t n_work, uint32_t n_parts, uint32_t n_groups,
                            uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, uint32_t kv_dim,
                            const void* pool, size_t pool_bytes,
                            void* workspace, size_t ws_bytes, void* stream, char* err, size_t errlen);

/* Split-KV partials without the final merge (long-context decode sharded over
 * GPUs).  Keys [t_begin, t_end) of one layer; writes per query head
 * ml[2*hh] = (m, l) and o[hh*head_dim ..] = unnormalised sum, where
 * m = max_t(score_t * log2(e)), l = sum_t 2^(score_t*log2(e) - m),
 * o = sum_t 2^(...) * v_t.  workspace as for yattn_decode_run with the plan
 * of a single item of t_end - t_begin keys (yattn_decode_partial_workspace_bytes). */
size_t yattn_decode_partial_workspace_bytes(uint32_t n_tokens, uint32_t n_heads,
                                            uint32_t n_kv_heads, uint32_t head_dim);
int yattn_decode_partial(float* ml, float* o, const float* q, const uint16_t* kcache,
                         const uint16_t* vcache, uint32_t t_begin, uint32_t t_end,
                         uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, uint32_t kv_dim,
                         void* workspace, size_t ws_bytes, void* stream, char* err, size_t errlen);

/* Merges n_parts partial sets laid out [n_parts][n_heads] (ml: 2 floats each,
 * o: head_dim floats each) into out[n_heads*head_dim]; gate as in
 * YattnDecodeItem.  Parts with l == 0 (empty shards) are skipped. */
int yattn_merge_partials(float* out, const float* ml, const float* o, uint32_t n_parts,
                         uint32_t n_heads, uint32_t head_dim, const float* gate,
                         void* stream, char* err, size_t errlen);

/* Same merge over packed parts: part s is parts[s*n_heads*(2+head_dim) ...],
 * its (m, l) pairs [n_heads][2] followed by its o [n_heads][head_dim] -- the
 * layout one all-gather of every rank's (ml, o) payload produces.  No
 * reference counterpart: the reference has no split-KV path. */
int yattn_merge_partials_packed(float* out, const float* parts, uint32_t n_parts,
                                uint32_t n_heads, uint32_t head_dim, const float* gate,
                                void* stream, char* err, size_t errlen);

/* ---- split-KV exchange over peer memory (long-context decode on 1..8 GPUs) ----
 * One process per GPU.  Each rank allocates a receive area
 * (yattn_exchange_area_alloc: cudaMalloc'd, zeroed) and maps every peer's area
 * through CUDA IPC (yattn_ipc_handle on the owner, 64-byte handles passed by
 * the caller's own transport, yattn_ipc_open on the others).
 * yattn_exchange_merge, after yattn_decode_partial wrote this rank's (ml, o):
 * stores them into every rank's area over NVLink (stores only, no peer loads),
 * raises this rank's per-head flags there (release, system scope), waits
 * (bounded by wait_limit_ns, 0 = 2 s) for every rank's flags in the local area
 * and merges all parts into out[n_heads*head_dim] (x sigmoid(gate) if gate).
 * A head whose parts all have l == 0 (every shard empty) gets 0.  If a rank's
 * flags do not arrive in time, yattn_device_status reads 401, out is NaN and
 * the areas' epochs are out of step: free and re-create them before another
 * call.  areas[r] is rank r's area as mapped in this process; areas[rank]
 * is the local one.  All ranks must make the same sequence of calls.  No
 * reference counterpart: the reference has no multi-GPU attention. */
size_t yattn_exchange_area_bytes(uint32_t world, uint32_t n_heads, uint32_t head_dim);
int yattn_exchange_area_alloc(uint32_t world, uint32_t n_heads, uint32_t head_dim, void** area_out,
                              char* err, size_t errlen);
int yattn_exchange_area_free(void* area, char* err, size_t errlen);
int yattn_ipc_handle(const void* area, void* handle_out /* 64 bytes */, char* err, size_t errlen);
int yattn_ipc_open(const void* handle /* 64 bytes */, void** ptr_out, char* err, size_t errlen);
int yattn_ipc_close(void* ptr, char* err, size_t errlen);
int yattn_exchange_merge(const float* ml, const float* o, void* const* areas, uint32_t world,
                         uint32_t rank, uint32_t n_heads, uint32_t head_dim, float* out,
                         const float* gate, uint64_t wait_limit_ns, void* stream, char* err,
                         size_t errlen);

/* One rank's step of a decode split over the GPUs, in two launches: the
 * partial decode of keys [k_begin, k_end) of this rank's cache, then one kernel
 * that merges this GPU's splits per head and exchanges the merged heads with
 * every rank through the receive areas (as yattn_exchange_merge does), so every
 * rank's out[n_heads*head_dim] holds the whole range's attention (x
 * sigmoid(gate) if gate).  k_begin == k_end (an empty shard) is allowed.
 * workspace: NULL (the per-device workspace) or yattn_decode_partial's.  Same
 * wait bound, timeout status (401, NaN output) and call discipline as
 * yattn_exchange_merge.  No reference counterpart: the reference has no
 * multi-GPU attention. */
int yattn_decode_exchange(const float* q, const uint16_t* kcache, const uint16_t* vcache,
                          uint32_t k_begin, uint32_t k_end, uint32_t n_heads, uint32_t n_kv_heads,
                          uint32_t head_dim, uint32_t kv_dim, void* const* areas, uint32_t world,
                          uint32_t rank, float* out, const float* gate, uint64_t wait_limit_ns,
                          void* workspace, size_t ws_bytes, void* stream, char* err, size_t errlen);

/* The new token's k and v of one item (device pointers, fp32, n_kv_heads*head_dim
 * each; k not yet rotated). */
typedef struct YattnDecodeNewRow {
    const float* k;
    const float* v;
} YattnDecodeNewRow;

/* yattn_decode_run_pooled with the decode step's RoPE and KV store fused into the
 * attention kernel: engine.c:1052-1072 (and 921-934 for qwen35's M-RoPE) for every
 * item in the same launch as its attention.  Each item's q is read unrotated (and
 * left as it is) and rotated at the item's pos; rows_dev[i] (same order as the
 * items) holds the new token's k and v: k is rotated, both are rounded with the
 * engine's f32_to_f16 and written into cache row pos of the item's K and V, and
 * the attention over keys 0..pos uses those fp16 values.  In the CTA of the split
 * that ends at pos, a warp of its own writes the row into the cache before that
 * split's last tile is copied; the rest of the cache is only read.  Row pos of an
 * item must lie inside the pool (else device status 103 and nothing is written).
 * rope_kind / n_rope_dims / theta as in yattn_rope_store_kv (no QK-norm here:
 * with QK-norm, run yattn_rope_store_kv first).  The plan, pool and workspace are
 * yattn_decode_plan_pooled's. */
int yattn_decode_run_pooled_rope(const YattnDecodeItem* items_dev, const YattnDecodeNewRow* rows_dev,
                                 const YattnDecodeWork* work_dev, uint32_t n_work, uint32_t n_parts,
                                 uint32_t n_groups, uint32_t n_heads, uint32_t n_kv_heads,
                                 uint32_t head_dim, uint32_t kv_dim, const void* pool, size_t pool_bytes,
                                 int rope_kind, uint32_t n_rope_dims, float theta, void* workspace,
                                 size_t ws_bytes, void* stream, char* err, size_t errlen);

/* Error-returning form of cuda_k_attn_decode with an explicit stream and gate. */
int yattn_attn_decode(float* att_out, const float* q, const uint16_t* kcache,
                      const uint16_t* vcache, const float* gate, uint32_t pos,
                      uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, uint32_t kv_dim,
                      void* stream, char* err, size_t errlen);

/* flags of yattn_attn_prefill: every q value is exactly an fp16 value (q built
 * from fp16 data).  The kernel then multiplies q's hi plane alone (no lo plane,
 * three TMEM score buffers instead of two): faster, with the same results for
 * such q.  It checks the claim; a q value that is not an fp16 value sets
 * yattn_device_status to 202 and that tile runs on the hi plane only. */
#define YATTN_PREFILL_Q_F16 1u

/* Error-returning form of cuda_k_attn_prefill with an explicit stream, the
 * qwen35 output gate (gate rows laid out like q, or NULL; engine.c:958-960) and
 * flags (0, or YATTN_PREFILL_Q_F16). */
int yattn_attn_prefill(float* att_out, const float* q, const uint16_t* kcache,
                       const uint16_t* vcache, const float* gate, uint32_t pos_start, uint32_t B,
                       uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, uint32_t kv_dim,
                       uint32_t q_stride, uint32_t flags, void* stream, char* err, size_t errlen);

/* Allocation-free form of yattn_attn_decode.  No counterpart in the reference:
 * it exists for callers that cannot call cudaMalloc while decoding (a serving
 * loop held to a device-memory budget fixed up front, or a host thread that
 * must not re-enter the allocator) and cannot hand the library a workspace.
 * The split-KV scratch lives in a fixed 4 MiB static device array that every
 * GPU loading this library holds until exit; a query whose split partials do
 * not fit (many splits at head_dim 256 with 8 query heads per kv head) is
 * rejected with an error naming the bytes needed.  The first call on a device
 * looks up the array's device address (no allocation), so make that first
 * call before any stream capture; after cudaDeviceReset() that address is
 * stale and this entry must not be called again in the process.  Every call on
 * a device shares the array and clears what must start at zero (the merge
 * counters); calls that overlap on the GPU (other streams or host threads) race
 * on it and must be serialised by the caller.  Device-side failures (a bounded
 * wait that gave up, a misaligned gate) are kept in the array's status word
 * until yattn_device_status reads and clears them.  Same arguments, results and
 * errors as yattn_attn_decode otherwise. */
int yattn_attn_decode_noalloc(float* att_out, const float* q, const uint16_t* kcache,
                              const uint16_t* vcache, const float* gate, uint32_t pos,
                              uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                              uint32_t kv_dim, void* stream, char* err, size_t errlen);

/* Pre-allocates the per-device workspace the drop-in entry points use, so no
 * allocation happens inside a decode step (the shim's bind-time workspace). */
int yattn_reserve(size_t bytes, char* err, size_t errlen);

/* Error-returning KV store (engine f32_to_f16 rounding), B rows at pos_start. */
int yattn_store_kv(uint16_t* kcache, uint16_t* vcache, const float* k, const float* v,
                   uint32_t pos_start, uint32_t B, uint32_t kv_dim, void* stream,
                   char* err, size_t errlen);

/* -------------------------------------------- Gated DeltaNet (qwen35)
 * State S: fp32 [n_vheads][hv][hk] per sequence (row j = v index, row stride
 * hv), updated in place.  v-head h reads k-head h % num_k_heads.  Supported:
 * hk == hv == 128; 16-byte aligned S, q, k, v, out, norm_w, z. */

/* Same argument order and meaning as gdn_state_update (inference/include/matvec.h:35-37,
 * inference/core/matvec.c:975-1004), on device pointers, legacy default stream:
 * one token, decay e^gate[h], delta rule with beta[h], out = S q / sqrt(hv). */
void cuda_k_gdn_state_update(float* S, float* out, const float* q, const float* k,
                             const float* v, const float* gate, const float* beta,
                             uint32_t num_k_heads, uint32_t hk, uint32_t n_vheads, uint32_t hv);

/* Batched single-token update of n_seqs independent sequences (engine.c:826-852):
 * S [n_seqs][n_vheads][hv][hk]; q,k [n_seqs][num_k_heads*hk]; v,out,z
 * [n_seqs][n_vheads*hv]; gate,beta [n_seqs][n_vheads].  With norm_w ([hv])
 * and z, out gets the rmsnorm_gated epilogue (matvec.c:1007-1021) per v-head. */
int yattn_gdn_decode(float* S, float* out, const float* q, const float* k, const float* v,
                     const float* gate, const float* beta, uint32_t n_seqs, uint32_t num_k_heads,
                     uint32_t hk, uint32_t n_vheads, uint32_t hv, const float* norm_w,
                     const float* z, float eps, void* stream, char* err, size_t errlen);

/* The GDN layer's inputs between its projections and the state update, for
 * T tokens of each of n_seqs sequences (engine.c:785-821, token by token on
 * the CPU): beta = sigmoid(beta_in), gate = softplus(alpha + ssm_dt) * ssm_a;
 * the causal depthwise conv1d of the projection over the kwidth-row delay line
 * (conv1d_update, matvec.c:956-967) and silu; the q / k / v split with
 * l2norm_inplace (matvec.c:941-948) of every q and k head.  One launch.
 *   qkv        [n_seqs][T][conv_chan]   projection (read only)
 *   conv_state [n_seqs][kwidth][conv_chan]  delay line, newest row last; updated
 *   conv_w     [conv_chan][kwidth]      fp32 taps (the GGUF layout)
 *   alpha, beta_in [n_seqs][T][n_vheads]; ssm_dt, ssm_a [n_vheads]
 *   q, k [n_seqs][T][num_k_heads*hk]; v [n_seqs][T][n_vheads*hv];
 *   gate, beta [n_seqs][T][n_vheads]: the layouts yattn_gdn_decode /
 *   yattn_gdn_prefill read.
 * conv_chan must be 2*num_k_heads*hk + n_vheads*hv; hk, hv <= 256; kwidth <= 8.
 * Operation order as the reference (fp32, no contraction); expf / log1pf are
 * the device's. */
int yattn_gdn_inputs(const float* qkv, float* conv_state, const float* conv_w, const float* alpha,
                     const float* beta_in, const float* ssm_dt, const float* ssm_a, float* q, float* k,
                     float* v, float* gate, float* beta, uint32_t n_seqs, uint32_t T,
                     uint32_t conv_chan, uint32_t kwidth, uint32_t num_k_heads, uint32_t hk,
                     uint32_t n_vheads, uint32_t hv, float eps, void* stream, char* err, size_t errlen);

/* T tokens of each of n_seqs sequences in order (the engine's qwen35 prefill,
 * engine.c:723-734, calls gdn_state_update once per token).  Per-token rows as
 * in yattn_gdn_decode, token t of sequence s at row s*T + t.  Runs the chunked
 * form (64-token chunks, tensor cores, fp32 state); the library grows a
 * per-device scratch of about (num_k_heads*64 + n_vheads*32.25) KiB per
 * 64 tokens per sequence on first use. */
int yattn_gdn_prefill(float* S, float* out, const float* q, const float* k, const float* v,
                      const float* gate, const float* beta, uint32_t n_seqs, uint32_t T,
                      uint32_t num_k_heads, uint32_t hk, uint32_t n_vheads, uint32_t hv,
                      const float* norm_w, const float* z, float eps, void* stream,
                      char* err, size_t errlen);

/* The same prefill token by token in the reference's operation order (one
 * recurrent kernel, no scratch).  No reference counterpart beyond
 * gdn_state_update itself; kept as the GPU cross-check of the chunked form. */
int yattn_gdn_prefill_recurrent(float* S, float* out, const float* q, const float* k,
                                const float* v, const float* gate, const float* beta,
                                uint32_t n_seqs, uint32_t T, uint32_t num_k_heads, uint32_t hk,
                                uint32_t n_vheads, uint32_t hv, const float* norm_w,
                                const float* z, float eps, void* stream, char* err, size_t errlen);

/* ------------------------------------------------ linear layers (decode glue)
 * y = W x for the engine's weight formats, W row-major [out][in]:
 *   Q4_K: 144-byte blocks of 256 weights (fp16 d, dmin; 12 bytes of 6-bit
 *         scales/mins; 128 bytes of nibbles), in % 256 == 0;
 *   fp16: [out][in] uint16_t.
 * x fp32 [B][in], y fp32 [B][out] (token t at row t).  Every weight byte is
 * read once per 4 tokens; fp32 accumulation with x kept fp32.  x and a Q4_K w
 * must be 16-byte aligned; fp16 takes any in and alignment (a slower path
 * unless in % 8 == 0 and both are 16-byte aligned).  Returns 0 or -1 + err. */
int yattn_gemv_q4k(float* y, const uint8_t* w, const float* x, uint32_t out, uint32_t in, uint32_t B,
                   void* stream, char* err, size_t errlen);
int yattn_gemv_f16(float* y, const uint16_t* w, const float* x, uint32_t out, uint32_t in, uint32_t B,
                   void* stream, char* err, size_t errlen);
/* One token through n (1..4) Q4_K matrices that read the same x, in one launch:
 * y[i][0..out[i]) = W_i x for the engine's q, k, v (or gate, up) projections,
 * which cuda_fwd.c:94-168 issues as separate cuda_k_gemv_q4k calls on the same
 * normalised hidden state.  y, w and out are host arrays of n entries; every
 * W_i is [out[i]][in], in % 256 == 0, 16-byte aligned, as is x.  Each y[i]
 * equals yattn_gemv_q4k(y[i], w[i], x, out[i], in, 1) bit for bit.  Returns 0
 * or -1 + err. */
int yattn_gemv_q4k_multi(uint32_t n, float* const* y, const uint8_t* const* w, const uint32_t* out,
                         const float* x, uint32_t in, void* stream, char* err, size_t errlen);

/* Drop-ins with the reference's names and signatures (cuda_kernels.h; kernels
 * cuda_kernels.cu:36-249), legacy default stream.  The f16 pair accepts the
 * reference's cuBLAS handle and fp16 x scratch and uses neither: x stays fp32
 * (the reference's cuBLAS path rounds x to fp16). */
int cuda_k_gemv_q4k(float* y, const uint8_t* w, const float* x, uint32_t out, uint32_t in,
                    char* err, size_t errlen);
int cuda_k_gemm_q4k(float* y, const uint8_t* w, const float* x, uint32_t out, uint32_t in,
                    uint32_t B, char* err, size_t errlen);
int cuda_k_gemv_f16(void* cublas, float* y, const uint16_t* w, const float* x, uint16_t* xf16,
                    uint32_t out, uint32_t in, char* err, size_t errlen);
int cuda_k_gemm_f16(void* cublas, float* y, const uint16_t* w, const float* x, uint16_t* xf16,
                    uint32_t out, uint32_t in, uint32_t B, char* err, size_t errlen);

/* ------------------------------------------------ session KV file (device KV)
 * The engine's session KV file (sess_kv_save / sess_kv_load, cache.c:174-247)
 * written from and read into a device KV blob in the engine's layout:
 * 2*n_blocks + 1 regions of max_seq rows x kv_dim fp16 (engine.c:261), block
 * l in 1..n_blocks using K region l and V region n_blocks + l.  The file holds
 * the first pos rows of those regions and is byte for byte the reference's, so
 * either side can read the other's files.  Rows move through pinned staging
 * buffers, device copies overlapping the file I/O.  Returns 0, or -1 with a
 * message (a load refuses a file of another n_blocks / kv_dim / max_seq or
 * with pos > max_seq, like the reference).  Both calls return after the
 * stream has finished the copies. */
int yattn_sess_kv_save(const uint16_t* kv_dev, uint32_t n_blocks, uint32_t kv_dim, uint32_t max_seq,
                       uint32_t pos, const char* path, void* stream, char* err, size_t errlen);
int yattn_sess_kv_load(uint16_t* kv_dev, uint32_t n_blocks, uint32_t kv_dim, uint32_t max_seq,
                       const char* path, uint32_t* pos, void* stream, char* err, size_t errlen);

/* ------------------------------------------------ seeded input generator
 * Deterministic on every device and bit-identical to the CPU restatement in
 * the test oracle: splitmix64 (platform.c:411-417) draws, Box-Muller with
 * IEEE-exact double arithmetic, the engine's f32_to_f16. */

enum { YATTN_GEN_F32 = 0,        /* float out */
       YATTN_GEN_F16 = 1,        /* uint16 fp16 bits (engine rounding) */
       YATTN_GEN_F32_F16 = 2,    /* float out, value rounded through fp16 */
       YATTN_GEN_F32_BF16 = 3 }; /* float out, value truncated to bf16 */

/* n_rows rows of n_heads*head_dim values: value j of row r is the
 * ((first_row + r)*n_heads*head_dim + j)-th N(0,1) draw of stream `seed`,
 * times scale; with rope != 0 the qwen half-split rotation at position
 * pos0 + r (angle (pos0+r)*theta^(-2i/head_dim)) is applied; then converted
 * per out_kind and stored at dst + r*row_stride elements. */
int yattn_gen_rows(void* dst, int out_kind, size_t row_stride, size_t n_rows,
                   uint32_t n_heads, uint32_t head_dim, uint64_t seed, uint64_t first_row,
                   double scale, int rope, uint32_t pos0, double theta,
                   void* stream, char* err, size_t errlen);

/* GDN gates: gate[i] = -softplus(z_a), beta[i] = sigmoid(z_b), z the
 * (first+i)-th draws of streams seed_a / seed_b. */
int yattn_gen_gdn_gates(float* gate, float* beta, uint64_t seed_a, uint64_t seed_b,
                        uint64_t first, size_t n, void* stream, char* err, size_t errlen);

/* GDN q/k rows: bf16(N(0,1)) then l2norm_inplace (matvec.c:942-949) per head. */
int yattn_gen_gdn_qk(float* dst, uint64_t seed, uint64_t first_row, size_t n_rows,
                     uint32_t n_heads, uint32_t head_dim, float eps,
                     void* stream, char* err, size_t errlen);

/* FNV-1a 64 over n bytes of device memory, computed in 1 MiB blocks
 * (a checksum of block checksums; equals the oracle's blockwise hash). */
int yattn_checksum(const void* data, size_t n, uint64_t* out_host, void* stream,
                   char* err, size_t errlen);

#ifdef __cplusplus
}
#endif
#endif /* YLLM_ATTN_SM100_H */
