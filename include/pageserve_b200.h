/*
 * pageserve_b200 — C ABI of the B200-native (sm_100a) decode-step hot path.
 *
 * Plain pointers and sizes only. Every pointer argument named *_dev is a CUDA
 * device pointer on the current device; `stream` is a cudaStream_t (pass the
 * caller's current stream, e.g. torch.cuda.current_stream().cuda_stream).
 * Calls are asynchronous with respect to the host unless stated otherwise.
 *
 * Return value: PS_OK (0) or a PS_ERR_* code; ps_last_error() then returns a
 * human-readable message (thread-local). Host-side validation runs before any
 * launch, so an error return means nothing was launched. Kernels never trap:
 * device-side range violations (a block id outside the pool, a token id
 * outside the vocabulary) skip the access and are recorded in a per-device
 * status word read by ps_device_status().
 *
 * Layouts (row-major, innermost last):
 *   KV cache       [num_blocks][block_size][num_kv_heads][head_dim]   (one layer)
 *   block tables   int32 [num_seqs][max_blocks_per_seq]
 *   q / attention  [tokens][num_q_heads][head_dim]
 *   int8 weight    int8 [N][K] with float32 scale [N]  (per output channel)
 *   activations    [M][K]
 *
 * The reference these entry points replace is Rakshit-gen/pageserve; each
 * declaration cites the reference function (file:line) whose behaviour it
 * reproduces.
 */
#ifndef PAGESERVE_B200_H_
#define PAGESERVE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define PS_API __attribute__((visibility("default")))
#else
#define PS_API
#endif

typedef struct CUstream_st* ps_stream_t; /* == cudaStream_t */

enum ps_dtype { PS_F32 = 0, PS_BF16 = 1, PS_F16 = 2, PS_I8 = 3 };

enum ps_status {
  PS_OK = 0,
  PS_ERR_INVALID = 1,     /* bad shape / dtype / null pointer  (Python: ValueError/TypeError) */
  PS_ERR_INDEX = 2,       /* block table too short, position out of range (Python: IndexError) */
  PS_ERR_CUDA = 3,        /* a CUDA runtime call failed (Python: RuntimeError) */
  PS_ERR_UNSUPPORTED = 4, /* shape/dtype this build has no kernel for (Python: NotImplementedError) */
  PS_ERR_DEVICE = 5,      /* the device status word holds an error (Python: RuntimeError) */
  PS_ERR_TIMEOUT = 6      /* a bounded device wait gave up (Python: TimeoutError) */
};

/* ---------------------------------------------------------------- library */

/* ABI version of this header (bumped on any signature change). */
PS_API int ps_abi_version(void);
/* Message of the last error returned on this host thread. */
PS_API const char* ps_last_error(void);
/* Number of kernels this library has launched in this process. */
PS_API uint64_t ps_launch_count(void);
/* Reads (and with clear != 0, clears) the current device's status word after
 * synchronising `stream`. *code receives 0 or a device error code
 * (1 block id, 2 slot, 3 token id, 4 wait timeout, 5 metadata). */
PS_API int ps_device_status(int* code, int clear, ps_stream_t stream);

/* ------------------------------------------------------- (a1) KV writes */

/* engine/paged_attention.py:62-79 (write_kv): copy k[i], v[i] (rows of
 * num_kv_heads*head_dim elements) to slot block_table[(start_pos+i)/bs]*bs +
 * (start_pos+i)%bs of k_cache / v_cache. Bit-exact (a copy). table_len is the
 * number of entries of block_table_dev; start_pos+num_tokens must fit in
 * table_len*block_size (else PS_ERR_INDEX, like the reference's list index). */
PS_API int ps_write_kv(void* k_cache_dev, void* v_cache_dev, const int32_t* block_table_dev, int table_len,
                int num_blocks, int block_size, int num_kv_heads, int head_dim, int dtype, int start_pos,
                int num_tokens, const void* k_dev, const void* v_dev, ps_stream_t stream);

/* Copy-on-write of KV blocks for prefix sharing (engine/prefix_cache.py:35-82
 * shares physical blocks between sequences; a sequence that continues from a
 * shared, partially filled block writes into a private copy instead). For each
 * of the n_pairs (src, dst) int32 pairs in pairs_dev, block dst of every layer
 * of both caches ([num_layers][num_blocks][block_size][num_kv_heads][head_dim],
 * the layout of engine/model.py:143-147) becomes a copy of block src. Ids
 * outside [0, num_blocks) skip the pair and are recorded in the status word. */
PS_API int ps_copy_kv_blocks(void* k_cache_dev, void* v_cache_dev, const int32_t* pairs_dev, int n_pairs,
                             int num_layers, int num_blocks, int block_size, int num_kv_heads, int head_dim,
                             int dtype, ps_stream_t stream);

/* Batched form of the slot mapping used by write_kv (engine/paged_attention.py:74-77)
 * for a step of several sequences: for sequence b with chunk tokens
 * [cu_q[b], cu_q[b+1]) starting at position start_pos[b], writes
 * positions[t] = start_pos[b] + (t - cu_q[b]) and
 * slots[t] = block_tables[b][pos / bs] * bs + pos % bs  (int32). */
PS_API int ps_build_slot_mapping(int32_t* positions_dev, int32_t* slots_dev, const int32_t* block_tables_dev,
                          int max_blocks_per_seq, const int32_t* cu_q_dev, const int32_t* start_pos_dev,
                          int num_seqs, int total_tokens, int num_blocks, int block_size, ps_stream_t stream);

/* ------------------------------------------- (a2-a5) paged attention */

/* Scratch bytes ps_paged_attention needs for these launch bounds (0 when
 * no split of the context is used). */
PS_API size_t ps_paged_attention_workspace_size(int num_seqs, int max_q_len, int max_ctx, int num_q_heads,
                                         int num_kv_heads, int head_dim);

/* engine/paged_attention.py:117-132 (paged_causal_attention_incremental),
 * batched over sequences, with gather_kv (:82-99) fused away: the kernel reads
 * the cache blocks in place through the block table. Sequence b's queries are
 * rows [cu_q[b], cu_q[b+1]) of q, at absolute positions start_pos[b] + i; its
 * context is start_pos[b] + (cu_q[b+1]-cu_q[b]) tokens; query row i attends to
 * key positions <= start_pos[b] + i (causal_attention_incremental, :16-50),
 * q head h reads kv head h / (num_q_heads/num_kv_heads), scale
 * 1/sqrt(head_dim). max_q_len / max_ctx are host upper bounds over the batch
 * (they size the grid; the kernel reads the true values on the device).
 * dtype PS_BF16 or PS_F16; head_dim 64 or 128. */
PS_API int ps_paged_attention(void* out_dev, const void* q_dev, const void* k_cache_dev, const void* v_cache_dev,
                       const int32_t* block_tables_dev, int max_blocks_per_seq, const int32_t* cu_q_dev,
                       const int32_t* start_pos_dev, int num_seqs, int total_q, int max_q_len, int max_ctx,
                       int num_blocks, int block_size, int num_q_heads, int num_kv_heads, int head_dim,
                       int dtype, void* workspace_dev, size_t workspace_bytes, ps_stream_t stream);

/* Allocation-free form of ps_paged_attention. No counterpart in the
 * reference: it serves callers that cannot call cudaMalloc (a plugin whose
 * host engine owns all device memory through its own pool, or a latency-
 * critical path where cudaMalloc's implicit synchronisation is not allowed).
 * Same inputs, outputs and semantics as ps_paged_attention, without the
 * workspace arguments: the split-context scratch is a static device array of
 * PS_ATTN_NOALLOC_SCRATCH_BYTES (8 MiB) that every GPU loading this library
 * holds until exit. A decode batch whose split partials exceed it is
 * rejected with PS_ERR_INVALID before any launch; a prefill batch (max_q_len x
 * q heads per kv head > 16) instead splits its key range into fewer pieces,
 * as many as fit. The first call on a device looks up the array's address
 * (cudaGetSymbolAddress) and keeps it for the life of the process; make it
 * before any stream capture, and reload the library after a device reset
 * (cudaDeviceReset), which may move the array. Calls that overlap on the GPU
 * share the array and race. This variant owns no status word: device-side
 * range errors (skipped accesses) and bounded-wait timeouts in the kernels go
 * unreported, so a caller that needs them uses ps_paged_attention. */
#define PS_ATTN_NOALLOC_SCRATCH_BYTES (8u << 20)
PS_API int ps_paged_attention_noalloc(void* out_dev, const void* q_dev, const void* k_cache_dev,
                                      const void* v_cache_dev, const int32_t* block_tables_dev,
                                      int max_blocks_per_seq, const int32_t* cu_q_dev, const int32_t* start_pos_dev,
                                      int num_seqs, int total_q, int max_q_len, int max_ctx, int num_blocks,
                                      int block_size, int num_q_heads, int num_kv_heads, int head_dim, int dtype,
                                      ps_stream_t stream);

/* ------------------------------------------------ (a6-a7) W8A16 linear */

/* engine/quantization.py:16-23 (quantize_per_channel) on the device:
 * scale[n] = max(max_k |w[n,k]|, 1e-8) / 127 (float32),
 * q[n,k] = clamp(round_half_even(w[n,k] / scale[n]), -127, 127). w is float32
 * or bf16 (dtype). Bit-exact against the reference for float32 input. */
PS_API int ps_quantize_per_channel(int8_t* q_dev, float* scale_dev, const void* w_dev, int dtype, int N, int K,
                            ps_stream_t stream);

/* engine/quantization.py:26-50 + F.linear (engine/model.py:168-190):
 * y[m,n] = scale[n] * sum_k x[m,k] * q[n,k] + bias[n] + residual[m,n]
 * (bias, residual optional: pass NULL). x, y, residual, bias in `dtype`
 * (PS_BF16/PS_F16 use the tensor-core path for M > 16; PS_F32 runs on CUDA
 * cores). Accumulates in float32. Equivalent to the reference's
 * dequantize-then-matmul with the dequantized weight kept in float32. */
PS_API size_t ps_w8a16_linear_workspace_size(int M, int N, int K);
PS_API int ps_w8a16_linear(void* y_dev, const void* x_dev, const int8_t* q_dev, const float* scale_dev,
                    const void* bias_dev, const void* residual_dev, int M, int N, int K, int dtype,
                    void* workspace_dev, size_t workspace_bytes, ps_stream_t stream);

/* The same W8A16 linear on a weight re-tiled once (ps_tile_int8_weight) into
 * contiguous 8 KB blocks [ceil(N/128)][ceil(K/64)][128][64] (zero padded):
 * every main-loop weight tile is one contiguous bulk copy instead of 128-256
 * separate 64-byte rows. Always runs on the tensor cores (bf16/f16). The
 * reference keeps q row-major (engine/quantization.py:33-34); the tiled copy
 * is this build's kernel-side layout of the same int8 values. */
PS_API size_t ps_tiled_int8_weight_bytes(int N, int K);
PS_API int ps_tile_int8_weight(int8_t* q_tiled_dev, const int8_t* q_dev, int N, int K, ps_stream_t stream);
PS_API size_t ps_w8a16_linear_tiled_workspace_size(int M, int N, int K);
PS_API int ps_w8a16_linear_tiled(void* y_dev, const void* x_dev, const int8_t* q_tiled_dev, const float* scale_dev,
                                 const void* bias_dev, const void* residual_dev, int M, int N, int K, int dtype,
                                 void* workspace_dev, size_t workspace_bytes, ps_stream_t stream);

/* Plain linear with a 16-bit weight (the unquantized lm_head,
 * engine/model.py:193): y[m,n] = sum_k x[m,k] * w[n,k] (+ bias). */
PS_API int ps_linear(void* y_dev, const void* x_dev, const void* w_dev, const void* bias_dev, const void* residual_dev,
              int M, int N, int K, int dtype, void* workspace_dev, size_t workspace_bytes, ps_stream_t stream);

/* Fused SwiGLU MLP input: out[m,i] = silu(gu[m,i]) * gu[m, I+i] where gu is
 * [gate | up] (engine/model.py:188-190). */
PS_API int ps_silu_mul(void* out_dev, const void* gate_up_dev, int M, int I, int dtype, ps_stream_t stream);

/* -------------------------------------------------- (a8-a9) norm / rope */

/* engine/model.py:29-34 (rms_norm) fused with the residual add of
 * engine/model.py:184,190: when residual_dev != NULL,
 * r = x + residual (rounded to dtype, stored to residual_out_dev when that is
 * non-NULL), else r = x; y = r * rsqrt(mean(r^2) + eps) * weight, float32
 * math, one rounding to dtype. */
PS_API int ps_rmsnorm(void* y_dev, void* residual_out_dev, const void* x_dev, const void* residual_dev,
               const void* weight_dev, float eps, int M, int H, int dtype, ps_stream_t stream);

/* engine/model.py:50-54 (apply_rope) with explicit per-token cos/sin rows
 * (T, D) in `dtype`: out = x*cos + rotate_half(x)*sin, x (T, H, D). */
PS_API int ps_apply_rope(void* out_dev, const void* x_dev, const void* cos_dev, const void* sin_dev, int T, int H,
                  int D, int dtype, ps_stream_t stream);

/* engine/model.py:168-178 fused: from the fused projection output
 * qkv[t] = [q (Hq*D) | k (Hkv*D) | v (Hkv*D)] (bias already added), rotate q
 * and k by position positions[t] (NeoX half rotation, cos/sin from the float32
 * table rope_cos/rope_sin [max_pos][D/2]) and write q to q_out (T, Hq, D), the
 * rotated k and v to slot slots[t] of the paged caches (write_kv,
 * engine/paged_attention.py:62-79). slots[t] < 0 skips the cache write. */
PS_API int ps_rope_qkv_write_kv(void* q_out_dev, void* k_cache_dev, void* v_cache_dev, const void* qkv_dev,
                         const int32_t* positions_dev, const int32_t* slots_dev, const float* rope_cos_dev,
                         const float* rope_sin_dev, int max_pos, int T, int num_q_heads, int num_kv_heads,
                         int head_dim, int num_slots, int dtype, ps_stream_t stream);

/* ------------------------------------------------------- (a10) the step */

/* F.embedding (engine/model.py:159): out[t] = table[ids[t]]. */
PS_API int ps_embedding(void* out_dev, const int64_t* ids_dev, const void* table_dev, int T, int H, int vocab,
                 int dtype, ps_stream_t stream);

/* Greedy next token, int(logits[row].argmax()) (server.py:51): first index of
 * the maximum of each row; logits (M, V) in dtype; out int32 [M]. */
PS_API int ps_argmax(int32_t* out_dev, const void* logits_dev, int M, int V, int ld, int dtype, ps_stream_t stream);

/* Gate/up projection fused with SwiGLU (engine/model.py:188-190:
 * F.silu(F.linear(x, gate_w)) * F.linear(x, up_w)): one tensor-core linear
 * over the row-interleaved weight [2I][K] (row 2i = gate row i, row 2i+1 =
 * up row i; int8 tiled with its per-row scale as ps_w8a16_linear_tiled, or
 * a 16-bit weight with w_tiled NULL), whose epilogue rounds gate and up to
 * dtype and writes y[m][i] = silu(gate) * up (float32 math, one rounding),
 * y (M, I) with N2 = 2I a multiple of 16. Same values as the gate|up linear
 * followed by ps_silu_mul. */
PS_API int ps_linear_swiglu(void* y_dev, const void* x_dev, const void* w_dev, int wdtype, const int8_t* w_tiled_dev,
                            const float* scale_dev, int M, int N2, int K, int dtype, ps_stream_t stream);

/* ---------------------------------------- (f) on-device token selection
 *
 * The reference picks each sequence's next token on the host
 * (int(logits[-1].argmax()), server.py:47-51, engine/runner.py:79-83);
 * ps_argmax is the batched greedy form. These add top-k and sampling.
 *
 * Top-k of each of M rows (row stride ld elements, V columns, dtype PS_F32 /
 * PS_BF16 / PS_F16): vals (float32, M x k) and idx (int32, M x k) sorted by
 * value descending, ties by index ascending (so k = 1 equals ps_argmax).
 * 1 <= k <= min(V, 1024). NaN ranks above +inf. */
PS_API int ps_topk(float* vals_dev, int32_t* idx_dev, const void* logits_dev, int M, int V, int ld, int k, int dtype,
                   ps_stream_t stream);
/* Sampling from each row's top-k (ps_topk's outputs): p_j proportional to
 * exp((v_j - v_0) / temperature), token = idx[first j whose cumulative p
 * exceeds u * sum(p)], u = uniforms_dev[row] in [0, 1). temperature > 0. */
PS_API int ps_sample_topk(int32_t* out_dev, const float* vals_dev, const int32_t* idx_dev, const float* uniforms_dev,
                          int M, int k, float temperature, ps_stream_t stream);

/* ------------------------------------- (e) fused tensor-parallel all-reduce
 *
 * Replaces the dist.all_reduce(partial, SUM) after each row-parallel linear
 * (engine/tensor_parallel.py:34-48, called for o_proj and down_proj) with a
 * push over peer memory: the linear's final writer stores its output tile
 * into every rank's receive buffer, and the next RMSNorm sums the ranks'
 * slots. One process per GPU; buffers are shared through CUDA IPC.
 *
 * Receive buffer (one per rank, zeroed by ps_comm_alloc):
 *   bytes [0, PS_COMM_CTRL_BYTES): u32 control words; set s in {0, 1} has its
 *     arrival flag at 4*s (written by every rank's producer), its consumed
 *     counter at 64 + 4*s and its producer CTA counter at 128 + 4*s (local);
 *     a 'broken' word at 192, set by the first wait that times out, makes
 *     every later wait on this buffer give up at once (re-zero to clear);
 *     from byte 1024, u32 [2 sets][256] row-block counters of the two-shot
 *     gather;
 *   then xg [2 sets][max_tokens][hidden] of dtype (the two-shot gathered
 *     residual stream), padded to 256 bytes;
 *   then slots [2 sets][world][max_tokens][hidden] of dtype (two-shot:
 *     [2 sets][world][max_tokens][hidden/world]).
 * The two sets alternate (o_proj -> set 0, down_proj -> set 1). Every wait is
 * bounded (a few seconds); on timeout PS_ERR_TIMEOUT-style code 4 is recorded
 * in the device status word (ps_device_status) and the kernel finishes. */
#define PS_COMM_CTRL_BYTES 4096
#define PS_COMM_MAX_WORLD 8

PS_API size_t ps_comm_buffer_bytes(int world, int max_tokens, int hidden, int dtype);
/* cudaMalloc + zero fill (IPC-shareable device memory). */
PS_API int ps_comm_alloc(void** buf_dev, size_t bytes);
PS_API int ps_comm_free(void* buf_dev);
/* Zero this rank's control words (after a timeout; every rank resets before
 * the next step). Synchronises `stream`. */
PS_API int ps_comm_reset(void* buf_dev, ps_stream_t stream);
/* cudaIpcGetMemHandle / cudaIpcOpenMemHandle on 64-byte opaque handles. */
PS_API int ps_ipc_get_handle(void* buf_dev, void* handle64_out);
PS_API int ps_ipc_open_handle(const void* handle64, void** peer_buf_out);
PS_API int ps_ipc_close(void* peer_buf);

/* Row-parallel linear with push (tensor_parallel.py:34-46, the local
 * product partial = x_shard @ W_shard.T): y = x @ W.T (* scale for int8 W,
 * per output row; no bias), M tokens, N = hidden, K = this rank's input
 * shard. Instead of a local output, every rank r's slot [set][rank] gets the
 * (M, N) result (rank_bufs[r]: rank r's receive buffer as mapped in this
 * process, rank_bufs[rank] this rank's own), then every rank's flag of `set`
 * is raised by one. Weight as ps_w8a16_linear_tiled (w_tiled != NULL, int8)
 * or ps_linear (16-bit W, w_tiled NULL); always the tensor-core kernel;
 * workspace from ps_w8a16_linear_tiled_workspace_size. */
PS_API int ps_linear_push(const void* x_dev, const void* w_dev, int wdtype, const int8_t* w_tiled_dev,
                          const float* scale_dev, int M, int N, int K, int dtype, void* const* rank_bufs, int world,
                          int rank, int set, int max_tokens, void* workspace_dev, size_t workspace_bytes,
                          ps_stream_t stream);

/* Two-shot form of ps_linear_push (the reduce-scatter half of the
 * all-reduce): columns [d * N/world, (d + 1) * N/world) of the (M, N) result
 * go to rank d only, into its slot [set][rank] of that column slice
 * ([max_tokens][N/world]); then every rank's flag of `set` is raised by one.
 * N/world must be a multiple of 128. Each rank sends (world-1)/world of its
 * partial instead of world-1 copies. Consumed by ps_tp_reduce_rmsnorm. */
PS_API int ps_linear_push_scatter(const void* x_dev, const void* w_dev, int wdtype, const int8_t* w_tiled_dev,
                                  const float* scale_dev, int M, int N, int K, int dtype, void* const* rank_bufs,
                                  int world, int rank, int set, int max_tokens, void* workspace_dev,
                                  size_t workspace_bytes, ps_stream_t stream);

/* The two-shot consumer (tensor_parallel.py:47 + engine/model.py:184-190):
 * this rank owns columns [rank * H/world, (rank + 1) * H/world). It waits for
 * every rank's scatter of `set`, sums the slots of its columns (float32, rank
 * order, rounded to dtype), adds x_old (the residual stream, row stride H;
 * NULL: none), stores the new residual slice into the gathered region
 * xg[set] of every rank's buffer (the all-gather, peer stores), then, once
 * all ranks' slices of a row block have arrived, writes y = rmsnorm(x) *
 * weight for whole rows (y = x when weight_dev is NULL). The new residual
 * stream stays in xg[set] (ps_comm_gathered_offset) for the next reduction's
 * x_old. phases: 3 (one launch per rank); a process emulating several ranks
 * on one GPU launches phase 1 for every rank, then phase 2 for every rank. */
PS_API int ps_tp_reduce_rmsnorm(void* y_dev, const void* x_old_dev, const void* weight_dev, float eps, int M, int H,
                                int dtype, void* const* rank_bufs, int world, int rank, int set, int max_tokens,
                                int phases, ps_stream_t stream);
/* Byte offset of xg[set] (the gathered residual stream, [max_tokens][hidden])
 * inside a receive buffer; 0 for invalid arguments. */
PS_API size_t ps_comm_gathered_offset(int world, int max_tokens, int hidden, int dtype, int set);

/* The consumer (tensor_parallel.py:47 + engine/model.py:184-190): waits until
 * `set`'s flag in this rank's buffer shows all `world` ranks, s = sum over
 * ranks of the slots (float32, rank order, rounded to dtype like the reduced
 * linear output). With weight_dev != NULL: x = x + s (rounded to dtype, in
 * place) and y = rmsnorm(x) * weight (ps_rmsnorm's math); with weight_dev
 * NULL: y = s (the plain all-reduce result; x unused). Re-arms the set. */
PS_API int ps_allreduce_rmsnorm(void* y_dev, void* x_dev, const void* weight_dev, float eps, int M, int H,
                                int dtype, void* buf_dev, int world, int set, int max_tokens, ps_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PAGESERVE_B200_H_ */
