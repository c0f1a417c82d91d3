/*
 * minitp_b200.h: C ABI of libminitp_b200.so, the sm_100a kernels behind the
 * minitp_b200 Python package (a drop-in for mini-TP's tensor-parallel
 * decode path).
 *
 * Conventions
 *   - Every entry point returns 0 on success or a negative MTPB_ERR_* code;
 *     mtpb_last_error() then describes the failure (per calling thread).
 *   - Pointers are device pointers unless stated otherwise. `stream` is a
 *     cudaStream_t (NULL = legacy default stream). Work is enqueued
 *     asynchronously on `stream`; nothing synchronises unless stated.
 *   - dtype: MTPB_F32 or MTPB_BF16 (the model's storage type). Accumulation
 *     is always fp32.
 *   - Matrices are row-major; weights use the PyTorch Linear layout
 *     [out_features, in_features].
 *   - Citations "ref: file:line" name the reference (mini-TP v0.4) interface
 *     an entry point replaces.
 */
#ifndef MINITP_B200_H_
#define MINITP_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MTPB_F32 0
#define MTPB_BF16 1

#define MTPB_OK 0
#define MTPB_ERR_INVALID (-1) /* bad argument or unsupported shape */
#define MTPB_ERR_CUDA (-2)    /* a CUDA runtime call failed */
#define MTPB_ERR_TIMEOUT (-3) /* a bounded wait on a peer ran out */
#define MTPB_ERR_DEVICE (-4)  /* a kernel recorded a bad position / token id */

/* ---------------------------------------------------------------- misc */
const char* mtpb_last_error(void);
int mtpb_version(void);
/* Programmatic dependent launch on (1, default) or off (0) for later launches. */
int mtpb_set_pdl(int enable);
/* Upper bound of weight bytes each GEMV CTA prefetches into L2 before it
 * waits for the previous kernel (default 4 MiB; 0 disables the prefetch). */
int mtpb_set_prefetch_cap(uint32_t bytes);
/* GEMV grid size in CTAs per SM (default 2, range [1, 8]); applies to later launches
 * and to graph captures made after the call. */
int mtpb_set_gemv_ctas_per_sm(int n);
/* bf16 projections with at least `rows` rows (default 64) run on the tensor-core
 * (tcgen05) GEMM instead of the GEMV kernel; a large value keeps them on the GEMV. */
int mtpb_set_tc_min_rows(int rows);
/* The same threshold for the projections of a kernel-chain decode step (one
 * row per batch row; default 8): from eight rows the CUDA-core GEMV runs short
 * of registers and is compute-bound, while the tensor cores stay HBM-bound.
 * No counterpart in the reference (a tuning switch of this library). */
int mtpb_set_tc_min_rows_decode(int rows);

/* Allow (1, default) or forbid (0) the CTA-pair tensor-core GEMM
 * (tcgen05 cta_group::2, 256 x 256 tiles on two SMs) for projections of at
 * least 256 rows; returns the previous setting. With 0, the single-CTA kernel
 * runs every tensor-core projection. No counterpart in the reference (a
 * tuning switch of this library). */
int mtpb_set_tc_pair(int enable);

/* Most K ranges per output tile of the single-CTA tensor-core GEMM (split K,
 * default 32; 1 turns it off); returns the previous value, -1 outside
 * [1, 64]. A projection of at most 64 rows whose output tiles fill at most
 * half of the SMs splits its K blocks into ranges (at least two 64-column blocks each, at
 * most one item per SM); partials go to a per-device fp32 workspace (about
 * 64 KB per SM, allocated on the first split call, which must not be under
 * graph capture) and are summed in range order by the last arriving CTA, so
 * results do not depend on timing. Split GEMMs of one device must not run
 * concurrently on two streams (they share that workspace). No counterpart in
 * the reference (a tuning switch of this library). */
int mtpb_set_tc_split(int max_splits);

/* Two-shot form of the model's AllReduce sites that are not fused into a
 * projection (prefill chunks, decode steps of many rows): reduce-scatter,
 * then all-gather (each rank reduces one column slice of every row and sends
 * the result to the others) for messages of at least min_bytes on at least
 * min_world ranks; smaller ones stay one-shot (every rank pushes its whole
 * partial to every peer). min_bytes < 0 turns it off, which is the default
 * (min_world 4): the extra flag round trip cost more than the copies saved
 * on the 7B prefill at TP=4. Both forms sum in rank order with the same
 * rounding, so results are identical. The standalone mtpb_allreduce* calls stay one-shot.
 * No counterpart in the reference (a tuning switch of this library). */
int mtpb_set_allreduce_two_shot(long long min_bytes, int min_world);

/* The form the library picks for a model AllReduce site of `bytes` bytes in
 * rows of H values on `world` ranks: the column slice width of the two-shot
 * form, or 0 for one-shot. No counterpart in the reference. */
int mtpb_allreduce_two_shot_cols(long long bytes, int H, int world, int dtype);

/* ------------------------------------------------------- communicator
 * Peer-memory communicator over NVLink (one per rank; TP group == world).
 * Replaces the torch.distributed process group used by the hot-path
 * collectives: ref: minitp/distributed/context.py:45-78 (init_context) and
 * minitp/distributed/collectives.py:147-214 (all_reduce, all_gather_dim0).
 * Setup: mtpb_comm_create on every rank, exchange the 64-byte handles from
 * mtpb_comm_ipc_handle (the host does this once, e.g. all_gather_object),
 * then mtpb_comm_open with all `world` handles in rank order. */
int mtpb_comm_create(int rank, int world, uint64_t slot_bytes, void** comm);
int mtpb_comm_ipc_handle(void* comm, void* handle_out /* 64 bytes, host */);
int mtpb_comm_open(void* comm, const void* handles /* world * 64 bytes, host */);
int mtpb_comm_destroy(void* comm);
/* Budget of every bounded wait on a peer flag, in nanoseconds (default 5 s). */
int mtpb_comm_set_timeout(void* comm, uint64_t timeout_ns);
/* Synchronises the device, then reads and returns the status word
 * (0 = healthy, else MTPB status bits: 1 timeout, 2 bad position, 4 bad token). */
int mtpb_comm_status(void* comm, uint32_t* status_out /* host */);
int mtpb_comm_clear_status(void* comm);
/* Device pointer to the int32 decode position read and advanced by the
 * captured decode step (mtpb_model_decode_step). */
int* mtpb_comm_pos_ptr(void* comm);
/* Enqueue a store of `pos` into that decode position (a one-thread kernel). */
int mtpb_comm_set_pos(void* comm, int pos, void* stream);
uint64_t mtpb_comm_slot_bytes(void* comm);
/* NVLink latency floor (measurement only; no counterpart in the reference):
 * this rank and `peer` bounce one 8-byte word `iters` times (both ranks make
 * the call, in the same order of calls); *ns_out (device memory) receives the
 * time of the last iters - warm round trips. One-way latency =
 * ns / (iters - warm) / 2. Waits are bounded by the communicator timeout
 * (status bit 1 on expiry). */
int mtpb_comm_pingpong(void* comm, int peer, int iters, int warm, unsigned long long* ns_out,
                       void* stream);

/* --------------------------------------------------------------- linear
 * y[M, N] = x[M, K] * w[N, K]^T (+ bias[N]), x rows `ldx` elements apart,
 * y rows `ldy` apart. ref: minitp/parallel/linear.py:58-59
 * (ColumnParallelLinear.forward, F.linear), linear.py:117 (RowParallel
 * partial), minitp/parallel/fused.py:57-61 (FusedQKV), embedding.py:87-90
 * (VocabParallelLMHead.forward). */
int mtpb_linear(const void* x, int ldx, const void* w, const void* bias, void* y, int ldy, int M,
                int N, int K, int dtype, void* stream);

/* act[M, I] = T(silu(T(gate)) * T(up)) with gate/up = x * w[2I, K]^T rows
 * [0, I) and [I, 2I). ref: minitp/parallel/fused.py:102-104 +
 * minitp/mlp.py:34-38. */
int mtpb_linear_swiglu(const void* x, int ldx, const void* w, void* act, int ldact, int M, int I,
                       int K, int dtype, void* stream);

/* Fused QKV projection + bias + RoPE + KV-cache append.
 * w: packed [q_rows + 2*kv_rows, K] as [q; k; v] (fused.py:26-74);
 * q_out [M, hq*hd] gets rotated q; k/v (rotated k, plain v) are written to
 * k_cache/v_cache [B, hkv, cap, hd] at slot cache_len + t (kv_cache.py:43-55).
 * Row m is token t = m % T of batch row m / T; its RoPE position is
 * rope_pos[t] (device int64) or cache_len + t when rope_pos is NULL.
 * cos/sin: fp32 [rope_len, hd] tables (rope.py:20-45).
 * ref: minitp/attention.py:58-69 with rope.py:47-64. */
int mtpb_qkv_rope(const void* x, int ldx, const void* w, const void* bias, void* q_out,
                  void* k_cache, void* v_cache, int B, int T, int hq, int hkv, int hd, int K,
                  int cap, int cache_len, const int64_t* rope_pos, const float* cos_tab,
                  const float* sin_tab, int rope_len, int dtype, void* comm, void* stream);

/* Grouped-query attention of rows q [B*T, hq*hd] against the cache
 * [B, hkv, cap, hd]: row (b, t) attends to positions [0, cache_len + t]
 * (decode: no mask; prefill: causal; chunked prefill: tril(cache_len)).
 * out [B*T, hq*hd]. scale = 1/sqrt(hd).
 * ref: minitp/attention.py:71-106 (GQA expand + F.scaled_dot_product_attention). */
int mtpb_attention(const void* q, const void* k_cache, const void* v_cache, void* out, int B, int T,
                   int hq, int hkv, int hd, int cap, int cache_len, int dtype, void* comm,
                   void* stream);

/* Same computation and arguments as mtpb_attention (without the
 * communicator), for callers that must not allocate device memory: hosts
 * whose caching allocator or memory budget owns every device byte, and
 * latency-bound loops that cannot afford the device-wide synchronisation
 * of cudaMalloc/cudaFree. It has no counterpart in the reference.
 *
 * mtpb_attention allocates its split-KV scratch on first use; this variant
 * keeps it in a fixed device array of MTPB_NOALLOC_SCRATCH_BYTES (4 MiB)
 * compiled into the library, which every GPU that loads the library holds
 * until the process exits. It calls no cudaMalloc or cudaFree. A shape whose
 * scratch would exceed the array fails with MTPB_ERR_INVALID and a message
 * giving the bytes it needs (decode shapes need well under 1 MiB; shapes
 * with B*T*hkv >= the SM count need none). The first call on each device
 * looks up the array's device address (cudaGetSymbolAddress) with that
 * device current; make that first call before any stream capture. All calls
 * on a device share the one array: calls that overlap on the GPU (on
 * different streams, or from several threads) race and must be ordered by
 * the caller. Each call clears the counters it needs at its start.
 *
 * `status` (device memory of the caller, may be NULL): a 32-bit word into
 * which the kernel ORs its error bits (the bits mtpb_comm_status reports:
 * 1 timeout, 2 bad position, 4 bad token). The caller reads it, and
 * clears it, whenever it chooses. With NULL the bits land in a word of the
 * fixed array that no call reads back, so device-side errors are then not
 * reported (the host checks above reject every input that sets one today). */
#define MTPB_NOALLOC_SCRATCH_BYTES (4u << 20)
int mtpb_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, void* out, int B,
                           int T, int hq, int hkv, int hd, int cap, int cache_len, int dtype,
                           uint32_t* status, void* stream);

/* RMSNorm: y = T(x * rsqrt(mean(x^2) + eps) * w) in fp32 math.
 * ref: minitp/layer.py:36-42. */
int mtpb_rmsnorm(const void* x, const void* w, void* y, int rows, int H, float eps, int dtype,
                 void* stream);

/* In-place SUM AllReduce of t [rows, H] over the communicator (one-shot
 * NVLink push, rank-ordered reduction: bit-identical on every rank).
 * ref: minitp/distributed/collectives.py:147-157 (all_reduce). */
int mtpb_allreduce(void* comm, void* t, int rows, int H, int dtype, void* stream);

/* Fused RowParallel reduce + bias + residual add + RMSNorm:
 *   out_res  = T(residual + T(T(sum_r partial_r) + bias))   (residual, bias optional)
 *   out_norm = RMSNorm(out_res) with gain                   (optional)
 * ref: minitp/parallel/linear.py:111-122 (RowParallelLinear.forward),
 * minitp/layer.py:64-65 (residual add), layer.py:36-42 (RMSNorm). */
int mtpb_allreduce_residual_rmsnorm(void* comm, const void* partial, const void* residual,
                                    const void* gain, const void* bias, void* out_res,
                                    void* out_norm, int rows, int H, float eps, int dtype,
                                    void* stream);

/* Vocab-parallel embedding: out[m] = table[ids[m] - vstart] if the id is in
 * [vstart, vend) else 0, then summed over ranks (exact: one non-zero term).
 * ref: minitp/parallel/embedding.py:44-50 (VocabParallelEmbedding.forward). */
int mtpb_embedding(void* comm, const int64_t* ids, const void* table, void* out, int M, int H,
                   int64_t vstart, int64_t vend, int64_t vocab, int dtype, void* stream);

/* Greedy argmax over vocab-sharded logits [M, V_local] (row stride ld):
 * packed fp32-key/id max per shard, one int64 per row and rank exchanged
 * over NVLink, ties to the lowest id; NaN loses when world > 1 and wins
 * (first NaN) when world == 1, as the reference does. ids_out: device
 * int64 [M], identical on every rank. scratch: device int64 [M * 64]
 * (M <= 64; no initialisation needed).
 * ref: minitp/parallel/embedding.py:118-172 (distributed_argmax, bitpack)
 * with collectives.py:185-214 (all_gather_dim0). */
int mtpb_argmax(void* comm, const void* logits, int M, int V_local, int64_t ld, int64_t vstart,
                int64_t* ids_out, int64_t* scratch, int dtype, void* stream);

/* ---------------------------------------------------------------- model
 * A TP Qwen2 decoder whose weights stay in caller-owned device tensors.
 * ref: minitp/layer.py:68-124 (TPQwen2ForCausalLM), minitp/attention.py,
 * minitp/mlp.py, minitp/generation.py:70-171. */
typedef struct {
  int dtype;
  int hidden;        /* H */
  int inter_local;   /* intermediate_size / tp */
  int n_layers;
  int hq_local;      /* query heads on this rank (after padding) */
  int hkv_local;     /* KV heads on this rank */
  int head_dim;
  int64_t vocab_start, vocab_end, vocab_size;
  float eps;
  const void* embed;       /* [vend - vstart, H] */
  const void* lm_head;     /* [vend - vstart, H] (the embedding when tied) */
  const void* final_norm;  /* [H] */
  const float* cos_tab;    /* fp32 [rope_len, head_dim] */
  const float* sin_tab;
  int rope_len;
} mtpb_model_desc;

typedef struct {
  const void* ln1;     /* input_layernorm [H] */
  const void* qkv_w;   /* [(hq + 2 hkv) hd, H] */
  const void* qkv_b;   /* [(hq + 2 hkv) hd] or NULL */
  const void* o_w;     /* [H, hq hd] */
  const void* ln2;     /* post_attention_layernorm [H] */
  const void* gu_w;    /* [2 inter_local, H] (gate; up) */
  const void* down_w;  /* [H, inter_local] */
} mtpb_layer_desc;

int mtpb_model_create(const mtpb_model_desc* desc /* host */, void* comm, void** model);
int mtpb_model_set_layer(void* model, int layer, const mtpb_layer_desc* desc /* host */);
/* Allocate scratch for up to max_rows token rows and KV capacity max_cap.
 * Call before capturing a CUDA graph (forward/decode_step never allocate
 * for sizes within the reservation). */
int mtpb_model_reserve(void* model, int max_rows, int max_cap);
int mtpb_model_destroy(void* model);

/* Forward of B x T tokens (ids device int64 [B*T]) at cache slots
 * [cache_len, cache_len + T): writes K/V into k_caches[l]/v_caches[l]
 * (host arrays of n_layers device pointers, each [B, hkv, cap, hd]) and
 * logits [B*T, V_local] (or [B, V_local] of the last token when last_only).
 * rope_pos: device int64 [T] or NULL (= slots). ref: minitp/layer.py:91-124. */
int mtpb_model_forward(void* model, const int64_t* ids, int B, int T, const int64_t* rope_pos,
                       int cache_len, void* const* k_caches, void* const* v_caches, int cap,
                       void* logits, int last_only, void* stream);

/* One greedy decode step for B rows, all state on the device: reads the
 * tokens from `tok` (device int64 [B]) and the position from
 * mtpb_comm_pos_ptr(), runs the model, selects the next tokens (distributed
 * argmax), writes them to tok and to out_ids[b, pos + 1] (row stride
 * ld_out; out_ids may be NULL), writes logits [B, V_local] when logits is
 * not NULL, and advances the position. Capturable in a CUDA graph.
 * ref: minitp/generation.py:119-130 + 161-170 (select_next, append,
 * decode_step of the fixed-length loop). */
int mtpb_model_decode_step(void* model, int64_t* tok, int B, void* const* k_caches,
                           void* const* v_caches, int cap, int64_t* out_ids, int ld_out,
                           void* logits, void* stream);

/* Number of kernel launches one mtpb_model_decode_step makes for B rows and
 * cache capacity `cap` with the current implementation setting (1 when the
 * megakernel runs it). */
int mtpb_model_decode_kernels(void* model, int B, int cap, int* launches);

/* Decode-step implementation: 0 (default) = the persistent megakernel (one
 * cooperative launch per token; used when B <= 8 and the shapes fit its
 * shared-memory plan), 1 = the chain of per-operation kernels. */
int mtpb_set_decode_impl(int impl);

/* Diagnostic: when `buf` (device uint64[16384]) is not NULL, later megakernel
 * launches record CTA 0's stage timeline there (%globaltimer ns): [0] start,
 * [1 + 12 l + e] the 12 stage events of layer l, [1 + 12 L ..] the LM-head and
 * selection events, [512 + s] the first weight copy of weight stage s,
 * [1000 ..] the phases of CTA 0's first attention item; the last CTA records
 * its stage events at [2048 + index], every CTA its layer-1 events at
 * [4096 + 1024 e + cta]. */
int mtpb_set_decode_trace(void* buf);

/* Megakernel weight stream: chunks of at most `chunk_kb` KiB for the layers
 * and `lm_chunk_kb` KiB for the LM head, in a shared-memory ring that takes
 * the rest of the block's shared memory. 0 (the default for both) chooses
 * them per shape: the LM head, and layers whose weights per CTA exceed two
 * ring-fulls, take half the ring (two chunks in flight); other layers 96
 * KiB for one batch row when the ring holds two, else 128.
 * `l2_flags` bit 0: stream weights with an L2 evict-first policy; bit 1:
 * prefetch the next layer's weight rows into L2 (default 3, both). */
int mtpb_set_decode_ring(int chunk_kb, int lm_chunk_kb, int l2_flags);

/* Megakernel: nanoseconds a thread sleeps between two polls of a data word
 * that has not arrived yet (0, the default: poll back to back). */
int mtpb_set_decode_spin(int backoff_ns);

/* Counter bumped by every mtpb_set_* call. A CUDA graph captured over this
 * library's calls keeps the settings in force at capture; a holder of such a
 * graph (the Python generation loop keeps one per shape) compares this value
 * with the one at capture and recaptures when it changed. No counterpart in
 * the reference. */
uint64_t mtpb_settings_epoch(void);

#ifdef __cplusplus
}
#endif

#endif /* MINITP_B200_H_ */
