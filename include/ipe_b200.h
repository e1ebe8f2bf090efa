/* ipe_b200: C-ABI of the B200 (sm_100a) kernels for the dense Qwen3 prefill/decode hot path.
 *
 * Plain pointers, sizes and a cudaStream_t passed as void*. No torch types. Every entry point
 * validates its arguments on the host, launches on the given stream without synchronising, and
 * returns an ipe_status; ipe_last_error() gives the message of the calling thread's last failure.
 * Pointers are device pointers unless stated. "bf16" buffers hold IEEE bfloat16, row-major and
 * contiguous unless a stride argument says otherwise.
 *
 * Each entry point names the reference code it replaces (mamadou-wane/inference-performance-
 * engineering, src/ipe/...). The reference has no native code: its "interface" for each step is a
 * PyTorch call inside ops.py / forward.py / engine.py, which these functions implement on the GPU.
 */
#ifndef IPE_B200_H
#define IPE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  IPE_OK = 0,
  IPE_ERR_ARGUMENT = 1,    /* bad pointer, size or shape: nothing was launched */
  IPE_ERR_UNSUPPORTED = 2, /* a shape the kernels are not built for */
  IPE_ERR_CUDA = 3,        /* a CUDA runtime / driver call failed */
  IPE_ERR_IO = 4,          /* a file could not be opened or read */
} ipe_status;

/* Linear-layer epilogues of ipe_gemm. */
typedef enum {
  IPE_EPI_STORE = 0,    /* C[m,n] = bf16(acc)                                        */
  IPE_EPI_RESIDUAL = 1, /* C[m,n] = bf16(R[m,n] + bf16(acc)); R may alias C         */
  IPE_EPI_SILU_MUL = 2, /* B rows interleaved in groups of 64 (gate, up); C[m,n/2] =
                           bf16(bf16(silu(bf16(gate))) * bf16(up))                  */
  IPE_EPI_LOGITS = 3,   /* C (fp32)[m,n] = float(bf16(acc))                          */
  IPE_EPI_PARTIAL = 4,  /* C (fp32)[m,n] = acc, unrounded: a tensor-parallel rank's part
                           of a sum that ipe_add_partial completes after the all-reduce */
} ipe_epilogue;

/* Device-resident step state: int64_t[IPE_STATE_WORDS]. Kernels given a non-null state read the
 * cache position and the sampling parameters from it instead of their host arguments, so a
 * captured decode step replays without host work. */
enum {
  IPE_STATE_POS = 0,         /* committed positions = position of the token being decoded   */
  IPE_STATE_STEP = 1,        /* index of the next sampled token in the history buffers      */
  IPE_STATE_SEED = 2,        /* Gumbel-max sampling seed                                     */
  IPE_STATE_TEMPERATURE = 3, /* float32 bits in the low word; 0 = greedy                    */
  IPE_STATE_WORDS = 8,
};

/* Rows of 64 gate rows followed by 64 up rows, the packing IPE_EPI_SILU_MUL and
 * ipe_rmsnorm_gate_up_silu expect. */
#define IPE_GATE_UP_GROUP 64
/* Floats per sampling partial record written by ipe_lm_head. */
#define IPE_PARTIAL_WORDS 8

/* ------------------------------------------------------------------ library */

const char* ipe_last_error(void);
int ipe_abi_version(void);
/* Reads (and with reset != 0 clears) the device error word of the current device: 0 = none,
 * 1 = token ID out of range, 2 = cache position out of range, 3 = a bounded wait timed out.
 * Synchronises the device. */
int ipe_device_error(int reset, int* out_code);

/* ------------------------------------------------------------------ elementwise */

/* RMSNorm over the last axis, fp32 statistics, two roundings at bf16.
 * Replaces ipe.ops.rms_norm (src/ipe/ops.py:23-33). dtype: 0 = bf16, 1 = fp32 (x, weight, out). */
int ipe_rmsnorm(const void* x, const void* weight, void* out, int64_t rows, int width, float eps,
                int dtype, void* stream);

/* out[i, :] = table[ids[i], :] (bf16). An ID outside [0, vocab) writes zeros and sets device
 * error 1. Replaces F.embedding in src/ipe/forward.py:125 and src/ipe/engine.py:106. */
int ipe_embed(const int64_t* ids, int64_t count, const void* table, int64_t vocab, int hidden,
              void* out, void* stream);

/* Per-head q_norm / k_norm (RMSNorm over head_dim 128), split-half RoPE from bf16 tables, and the
 * K/V cache append, for `batch` rows of `tokens` tokens at positions start..start+tokens-1 (from
 * state[IPE_STATE_POS] when state is non-null).
 *   qkv      bf16 [batch*tokens, (q_heads + 2*kv_heads) * 128]   (q | k | v per token)
 *   cos/sin  bf16 [>= start+tokens, 128] indexed by absolute position
 *   q_out    bf16 [batch, q_heads, tokens, 128]
 *   k/v      bf16 [batch, kv_heads, capacity, 128] (one layer of the cache)
 * Replaces src/ipe/forward.py:101-109 (qk_norm, apply_rotary, cache write; ops.py:36-63). */
int ipe_qk_norm_rope_append(const void* qkv, int batch, int tokens, int q_heads, int kv_heads,
                            const void* q_norm_weight, const void* k_norm_weight,
                            const void* cos_table, const void* sin_table, int start,
                            const int64_t* state, void* q_out, void* k_cache, void* v_cache,
                            int capacity, float eps, void* stream);

/* ------------------------------------------------------------------ decode linear layers
 * Weight-streaming kernels for batch 1..16 rows (one token each). Their weight operand is the
 * "decode tile" layout of a bf16 [out, in] matrix (out % 32 == 0, in % 128 == 0), built once by
 * ipe_decode_tiles: 8 KB tiles of 32 rows x 128 columns (for gate/up: 16 gate rows then the 16
 * matching up rows), 16-byte chunks swizzled, row-block-major, so every weight byte is streamed by
 * one contiguous bulk copy. One persistent CTA per SM streams its share of the tiles through a
 * shared-memory ring; when the reduction dimension is split across CTAs, partial tiles go to
 * `workspace` (ipe_decode_linear_workspace bytes, zero-filled before its first use; the kernels
 * leave its counters at zero, so one workspace serves every call on a stream). Launched with
 * programmatic dependent launch: a call's weight stream overlaps the end of the previous kernel. */

/* Writes the decode tiles of w [rows, in] (or, with w_up, of the gate/up pair w = gate_proj,
 * w_up = up_proj, each [rows, in]) into `tiles` (ipe_decode_tiles_bytes bytes). */
int ipe_decode_tiles(const void* w, const void* w_up, void* tiles, int rows, int in_features,
                     void* stream);
size_t ipe_decode_tiles_bytes(int rows, int in_features, int gate_up_pair);
size_t ipe_decode_linear_workspace(int batch, int weight_rows, int in_features);

/* qkv[b,:] = rms_norm(x[b,:]) @ w_qkv^T; w_qkv (decode tiles) rows are q_proj | k_proj | v_proj.
 * Replaces src/ipe/forward.py:100-103 (rms_norm + three F.linear). */
int ipe_rmsnorm_qkv(const void* x, const void* norm_weight, const void* w_qkv, void* qkv_out,
                    int batch, int hidden, int qkv_rows, float eps, void* workspace,
                    size_t workspace_bytes, void* stream);

/* x[b,n] = bf16(x[b,n] + bf16(a[b,:] . w[n,:])). Replaces the o_proj and down_proj residual
 * updates, src/ipe/forward.py:113 and :115. */
int ipe_linear_residual(const void* a, const void* w, void* x, int batch, int in_features,
                        int out_features, void* workspace, size_t workspace_bytes, void* stream);

/* act[b,j] = bf16(bf16(silu(bf16(g))) * bf16(u)), g / u = rms_norm(x[b]) . gate/up row j;
 * w_gate_up: the decode tiles of the (gate_proj, up_proj) pair. Replaces src/ipe/forward.py:114-115
 * (rms_norm, then ops.swiglu's gate/up/silu/mul, src/ipe/ops.py:104-106). */
int ipe_rmsnorm_gate_up_silu(const void* x, const void* norm_weight, const void* w_gate_up,
                             void* act_out, int batch, int hidden, int intermediate, float eps,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Tensor-parallel pieces (one rank of t holding a column shard of a row-parallel layer):
 * out (fp32) [b, n] = a[b, :] . w[n, :], unrounded, to be summed over the ranks (an all-reduce)
 * and then applied by ipe_add_partial. Replaces the rank's share of the o_proj / down_proj
 * products of src/ipe/forward.py:113, :115 under a Megatron split. */
int ipe_linear_partial(const void* a, const void* w, float* out, int batch, int in_features, int out_features,
                       void* workspace, size_t workspace_bytes, void* stream);
/* x[i] = bf16(x[i] + bf16(sum[i])) for i < count: the residual add of a layer whose product was
 * summed in fp32 over the ranks, rounded once as the unsplit layer rounds. */
int ipe_add_partial(void* x, const float* sum, int64_t count, void* stream);

/* Final RMSNorm of x rows (row b at x + b*x_row_stride elements), tied LM head (its decode
 * tiles), fp32 logits
 * (bf16-rounded then widened, as the reference), and per-block sampling partials
 * [ipe_lm_head_parts(vocab)][batch][IPE_PARTIAL_WORDS] for ipe_sample. temperature > 0 adds
 * Gumbel noise from (seed, position) to the sampling partials only.
 * Replaces src/ipe/engine.py:110-111 and the first pass of src/ipe/engine.py:28-41. */
int ipe_lm_head(const void* x, int64_t x_row_stride, const void* norm_weight, const void* embed_tiles,
                float* logits, float* partials, int batch, int hidden, int vocab, float eps,
                float temperature, uint64_t seed, const int64_t* state, void* stream);
int ipe_lm_head_parts(int vocab);
/* ipe_lm_head over a vocabulary shard: embed_tiles holds rows vocab_offset .. vocab_offset +
 * vocab_rows - 1 (vocab_offset a multiple of 32), logits is [batch, vocab_rows], and the records
 * carry global vocabulary IDs and Gumbel draws, so ranks' records gathered in order sample as the
 * unsharded head would (ipe_sample_records). */
int ipe_lm_head_shard(const void* x, int64_t x_row_stride, const void* norm_weight, const void* embed_tiles,
                      float* logits, float* partials, int batch, int hidden, int vocab_rows, int vocab_offset,
                      float eps, float temperature, uint64_t seed, const int64_t* state, void* stream);

/* Token and untempered log-probability per row from the partials: argmax (lowest ID on ties)
 * when temperature == 0, else Gumbel-max. Writes tokens[b*stride + step] and logprobs[...] with
 * step = state[IPE_STATE_STEP] (0 without state; the state's step then advances by 1), and
 * next_tokens[b] (nullable) for the next decode step. Replaces src/ipe/engine.py:28-41. */
int ipe_sample(const float* partials, const float* logits, int batch, int vocab, float temperature,
               int64_t* state, int64_t* tokens, float* logprobs, int64_t stride,
               int64_t* next_tokens, void* stream);

/* ipe_sample from `parts` records alone (no logits): the chosen token's logit comes from the
 * records (the maximum for argmax, the carried logit for the Gumbel winner). For records gathered
 * from vocabulary shards; padding records (max -inf, sum 0) are neutral. */
int ipe_sample_records(const float* partials, int parts, int batch, float temperature, int64_t* state,
                       int64_t* tokens, float* logprobs, int64_t stride, int64_t* next_tokens, void* stream);

/* The same rule over a logits matrix [rows, vocab] (fp32) already in memory, any number of rows:
 * tokens[r], logprobs[r]. Gumbel noise is drawn from (seed, row, vocab id). Replaces
 * ipe.engine.sample (src/ipe/engine.py:28-41) for logits the caller holds. */
int ipe_sample_logits(const float* logits, int64_t rows, int vocab, float temperature, uint64_t seed,
                      int64_t* tokens, float* logprobs, void* stream);

/* ------------------------------------------------------------------ attention */

/* Split-KV flash-decode: one query token per row against keys 0..length-1 of the cache
 * (length = state[IPE_STATE_POS] + 1 when state is non-null), GQA (query head j reads KV head
 * j / (q_heads / kv_heads)), scale 128^-0.5, fp32 softmax.
 *   q bf16 [batch, q_heads, 128] -> out bf16 [batch, q_heads * 128]
 * workspace: ipe_decode_attention_workspace(batch, q_heads, capacity) bytes of device memory.
 * A device state whose position lies outside 0..capacity-1 makes the kernels read and write
 * nothing and sets the device error word to 2 (ipe_device_error).
 * Replaces ops.attention for decode steps (src/ipe/ops.py:78-101, causal=False). */
int ipe_decode_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                         int batch, int q_heads, int kv_heads, int capacity, int length,
                         const int64_t* state, void* workspace, size_t workspace_bytes,
                         void* stream);
size_t ipe_decode_attention_workspace(int batch, int q_heads, int capacity);

/* One decode step's attention straight from the QKV projection output: per-head q_norm / k_norm
 * and RoPE of the step's query and key (as ipe_qk_norm_rope_append), the K/V append at position
 * `start` (state[IPE_STATE_POS] when state is non-null), split-KV attention over positions
 * 0..position, and the merge of the chunks by the last chunk block of each (row, KV head).
 *   qkv bf16 [batch, (q_heads + 2*kv_heads) * 128] -> out bf16 [batch, q_heads * 128]
 * workspace: ipe_decode_attention_qkv_workspace bytes, zero-filled before first use (its arrival
 * counters return to zero after every call). The caches and the workspace must be 16-byte aligned
 * (K / V rows and the split records move by bulk copies into shared memory), else
 * IPE_ERR_ARGUMENT. Replaces src/ipe/forward.py:101-112 for a decode step
 * (qk_norm, apply_rotary, cache write, ops.attention). */
int ipe_decode_attention_qkv(const void* qkv, const void* q_norm_weight, const void* k_norm_weight,
                             const void* cos_table, const void* sin_table, int start,
                             const int64_t* state, void* k_cache, void* v_cache, void* out, int batch,
                             int q_heads, int kv_heads, int capacity, float eps, void* workspace,
                             size_t workspace_bytes, void* stream);
size_t ipe_decode_attention_qkv_workspace(int batch, int q_heads, int kv_heads, int capacity);

/* The same decode attention for callers that cannot allocate device memory: a host that gives a
 * plugin only its input and output buffers and keeps every other allocation to itself, or a loop
 * that must not call cudaMalloc / cudaFree because they can synchronise the device. It takes no
 * workspace and allocates nothing: the split partials go to a 2 MiB array the library declares
 * in device memory, which every GPU that loads the library holds until the process exits.
 * Limit: ipe_decode_attention_workspace(batch, q_heads, capacity) must be <= 2 MiB (for 16 query
 * heads: batch x capacity up to about 8,000 positions), else IPE_ERR_UNSUPPORTED and nothing runs.
 * A device state position outside 0..capacity-1 is handled as by ipe_decode_attention: nothing
 * is read or written and the device error word reads 2.
 * The first call on each device looks up the array's device address (cudaGetSymbolAddress, with
 * that device current); make that first call before any stream capture. All calls share the one
 * array and it keeps the last call's contents; nothing in it needs clearing, because a call only
 * reads the partial records it wrote itself. Calls whose executions overlap on the GPU (other
 * streams, other threads) race on the array and must be serialised by the caller.
 * No counterpart in the reference: this entry point exists only in this library. */
int ipe_decode_attention_static_scratch(const void* q, const void* k_cache, const void* v_cache,
                                        void* out, int batch, int q_heads, int kv_heads,
                                        int capacity, int length, const int64_t* state,
                                        void* stream);

/* Causal flash-attention over a prompt of `tokens` positions written at cache positions
 * 0..tokens-1.
 *   q bf16 [batch, q_heads, tokens, 128] -> out bf16 [batch, tokens, q_heads * 128]
 * Replaces ops.attention for a prompt (src/ipe/ops.py:78-101, causal=True). */
int ipe_prefill_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                          int batch, int q_heads, int kv_heads, int tokens, int capacity,
                          void* stream);

/* ------------------------------------------------------------------ tensor-core GEMM */

/* C = epilogue(A @ B^T): A bf16 [m, k], B bf16 [n, k] (both k-contiguous), tcgen05 MMA with
 * TMEM accumulators fed by TMA. n % 128 == 0, k % 64 == 0, pointers 16-byte aligned.
 * Replaces the prefill F.linear calls of src/ipe/forward.py:100-115 and the uncached LM head of
 * src/ipe/forward.py:145-152. */
int ipe_gemm(const void* a, const void* b, void* c, int m, int n, int k, int epilogue,
             const void* residual, void* stream);

/* ------------------------------------------------------------------ NVLink all-reduce
 * One-shot all-reduce of tensor-parallel fp32 parts over peer memory, fused with the residual add
 * (replaces the NCCL all-reduce + ipe_add_partial pair of a decode step). Each rank allocates one
 * communication region (ipe_comm_alloc, ipe_comm_bytes(slot_bytes) bytes, zero-filled), exchanges
 * its IPC handle (ipe_ipc_handle, 64 bytes) with the group, opens the peers' (ipe_ipc_open) and
 * keeps a device array of the world region pointers, its own at index `rank`. A layer's partial
 * product goes into this rank's slot (region + ipe_comm_slot_offset(slot, slot_bytes)); then
 * ipe_allreduce_residual sets x[i] = bf16(x[i] + bf16(sum over ranks of slot[i])), summing in rank
 * order so every rank gets the same bits. Consecutive calls must alternate slots 0 / 1, and every
 * rank must make the same calls in the same order. Waits for the peers are bounded (about 2 s;
 * then device error 3 is set and x is left unchanged). */
size_t ipe_comm_bytes(size_t slot_bytes);
size_t ipe_comm_slot_offset(int slot, size_t slot_bytes);
int ipe_comm_alloc(size_t bytes, void** ptr);
int ipe_comm_free(void* ptr);
int ipe_ipc_handle(const void* ptr, void* handle);
int ipe_ipc_open(const void* handle, void** ptr);
int ipe_ipc_close(void* ptr);
int ipe_allreduce_residual(void* x, int64_t count, const void* peers, int world, int rank, int slot,
                           size_t slot_bytes, void* stream);

/* ------------------------------------------------------------------ fp32 (plumbing) path
 * The reference at dtype float32 (TF32 disabled, src/ipe/forward.py:42-43): fp32 storage and fp32
 * FMA arithmetic, no bf16 rounding points, no tensor cores. Row-major fp32 operands; the RMSNorm
 * is ipe_rmsnorm with dtype 1 and sampling is ipe_sample_logits. */

/* C[m, n'] = epilogue(A[m, k] . W[n, k]^T) in fp32: store / residual (C = R + acc, R may alias C)
 * / logits (store); SiLU*up takes W = the gate/up rows interleaved in groups of IPE_GATE_UP_GROUP
 * (n = 2 * intermediate) and writes n' = n / 2 columns of silu(gate) * up. Replaces the fp32
 * F.linear calls of src/ipe/forward.py:100-115 and lm_logits (src/ipe/forward.py:145-152). */
int ipe_gemm_f32(const void* a, const void* w, void* c, int m, int n, int k, int epilogue, const void* residual,
                 void* stream);
/* out[i, :] = table[ids[i], :] (fp32); an ID outside [0, vocab) writes zeros and sets device
 * error 1. Replaces F.embedding (src/ipe/forward.py:125) at fp32. */
int ipe_embed_f32(const int64_t* ids, int64_t count, const void* table, int64_t vocab, int hidden, void* out,
                  void* stream);
/* ipe_qk_norm_rope_append at fp32 (qkv, norm weights, cos/sin tables, q_out and caches fp32; host
 * start only). Replaces src/ipe/forward.py:101-109 at fp32. */
int ipe_qk_norm_rope_append_f32(const void* qkv, int batch, int tokens, int q_heads, int kv_heads,
                                const void* q_norm_weight, const void* k_norm_weight, const void* cos_table,
                                const void* sin_table, int start, void* q_out, void* k_cache, void* v_cache,
                                int capacity, float eps, void* stream);
/* Causal attention in fp32: query t of q [batch, q_heads, tokens, 128] (position start + t) over
 * cache keys 0 .. start + t, GQA, scale 128^-0.5, fp32 softmax -> out [batch, tokens,
 * q_heads * 128]. A decode step is tokens = 1, start = its position. Replaces ops.attention
 * (src/ipe/ops.py:78-101) at fp32. */
int ipe_attention_f32(const void* q, const void* k_cache, const void* v_cache, void* out, int batch, int q_heads,
                      int kv_heads, int tokens, int capacity, int start, void* stream);

/* ------------------------------------------------------------------ whole decode step */

/* One decoder layer's operands for ipe_decode_step (device pointers, each 16-byte aligned; the
 * array lives in device memory, so the host entry point cannot check them). */
typedef struct {
  const void* input_layernorm;          /* bf16 [hidden]                                    */
  const void* post_attention_layernorm; /* bf16 [hidden]                                    */
  const void* q_norm;                   /* bf16 [128]                                       */
  const void* k_norm;                   /* bf16 [128]                                       */
  const void* qkv_tiles;                /* decode tiles of q_proj | k_proj | v_proj          */
  const void* o_tiles;                  /* decode tiles of o_proj                            */
  const void* gate_up_tiles;            /* decode tiles of the (gate_proj, up_proj) pair     */
  const void* down_tiles;               /* decode tiles of down_proj                         */
  void* k_cache;                        /* bf16 [batch_rows, kv_heads, capacity, 128]        */
  void* v_cache;
} ipe_layer_desc;

/* Everything one decode step reads and writes. Device pointers unless stated. */
typedef struct {
  int layers, hidden, intermediate, q_heads, kv_heads, vocab, capacity, batch;
  float eps;
  const ipe_layer_desc* layer_descs; /* device array of `layers` descriptors (16-byte aligned;
                                        copied into shared memory once per step)             */
  const void* embed;                 /* bf16 [vocab, hidden], row-major (the input embedding) */
  const void* lm_head_tiles;         /* decode tiles of the (tied) LM head                    */
  const void* final_norm;            /* bf16 [hidden]                                         */
  const void* cos_table;             /* bf16 [capacity, 128]                                  */
  const void* sin_table;
  int64_t* state;                    /* int64[IPE_STATE_WORDS]: position read, then advanced */
  int64_t* tokens;                   /* [batch] input IDs; the sampled IDs when sampling      */
  void* x;                           /* bf16 [batch, hidden] residual stream                  */
  void* qkv;                         /* bf16 [batch, (q_heads + 2 kv_heads) * 128]            */
  void* attn;                        /* bf16 [batch, q_heads * 128]                           */
  void* act;                         /* bf16 [batch, intermediate]                            */
  float* logits;                     /* fp32 [batch, vocab]                                   */
  float* partials;                   /* [ipe_lm_head_parts(vocab)][batch][IPE_PARTIAL_WORDS]  */
  void* workspace;                   /* ipe_decode_step_workspace bytes, zero-filled once     */
  size_t workspace_bytes;
  int64_t* history_tokens;           /* nullable: sample the next token into [b*stride+step] */
  float* history_logprobs;
  int64_t history_stride;
  uint64_t* trace;                   /* nullable: per-CTA phase timestamps, see below         */
  /* Tensor parallelism (tp_world > 1; tp_world 0 or 1 is one GPU). q_heads, kv_heads,
   * intermediate and vocab (LM-head rows, from vocab_offset) are then this rank's shard; the
   * weights, caches and tiles above are the shard's. o_proj and down_proj push fp32 parts into
   * every rank's communication region (tp_peers: device array of the tp_world region pointers,
   * ipe_decode_step_comm_bytes each, zero-filled once) as flagged 64-bit elements {value, epoch}, and the next
   * phase polls and sums them in rank order; each CTA's merge of its LM-head records goes to
   * every rank the same way and every rank samples the same token. No grid barrier follows a row-parallel phase. x_alt: a
   * second bf16 [batch, hidden] residual buffer. Needs hidden % 512 == 0 and the activations in
   * shared memory (the launch fails with a message when the batch is too large for that). */
  int tp_world, tp_rank;
  const void* tp_peers;
  void* x_alt;
  int vocab_offset;                  /* first vocabulary ID of this rank's LM-head rows        */
  int vocab_total;                   /* the full vocabulary (token IDs)                         */
  /* Bound of every spin-wait of the step (grid barriers, shared-memory copies, a peer's parts) in
   * nanoseconds; 0 means 2 s. A wait that runs out sets device error 3 (ipe_device_error), every
   * CTA leaves at its next wait, and the step neither samples nor advances state[IPE_STATE_POS]. */
  int64_t wait_limit_ns;
} ipe_decode_step_desc;

/* Step trace (when desc.trace is set): CTA c writes globaltimer nanoseconds to
 * trace[c * IPE_TRACE_WORDS(layers) + i]: i = 0 kernel start; for phase end j = 1 .. 5*layers+2
 * (embedding, then per layer after QKV, attention, o_proj, gate/up, down_proj, then the LM head;
 * a grid barrier, except after o_proj, down_proj and the LM head of a tensor-parallel step),
 * i = 5j-4 its arrival, 5j-3 its release (the same time without a barrier), and for the phase
 * that follows it: 5j-2 activations staged, 5j-1 first weight tile (attention: first item) ready,
 * 5j last weight tile ready (last item done); the second-to-last word the CTA's end of the LM
 * head, the last its exit (CTA 0: after sampling). Words of events that did not happen are left
 * as they were. The array needs ipe_decode_step_grid() * IPE_TRACE_WORDS(layers) words. */
#define IPE_TRACE_WORDS(layers) (25 * (layers) + 13)
int ipe_decode_step_grid(void);

/* One whole decode step (embedding, all layers, final norm, LM head, and the sampler when
 * history_tokens is set) as ONE persistent cooperative kernel, one CTA per SM: a producer warp
 * per SM streams every phase's decode tiles back to back with bulk copies, consumer warps meet at
 * bounded-spin grid barriers between phases. Reads the position from state[IPE_STATE_POS] and
 * advances it (and state[IPE_STATE_STEP] when sampling) at the end. Deterministic. Replaces
 * src/ipe/engine.py:84-111 (decode -> _step) and, with sampling, one iteration of
 * src/ipe/engine.py:137-147. */
int ipe_decode_step(const ipe_decode_step_desc* desc, void* stream);
/* Checkpoint loading. Reads `count` byte ranges [offsets[i], offsets[i] + sizes[i]) of file
 * paths[file_of[i]] (of `files` files) into device memory at destinations[i] (current device), in
 * chunks of at most staging_bytes taken in list order by `threads` (1..64) reader threads, each
 * with two pinned staging buffers of staging_bytes: a reader fills one buffer while the
 * host-to-device copy of the other (on `stream`) runs. Returns once every copy has finished.
 * IPE_ERR_IO when a file cannot be opened or read (ipe_last_error names it), IPE_ERR_ARGUMENT for
 * a range outside its file. Replaces the per-tensor mmap -> .to(dtype) -> .to(device) copies of
 * src/ipe/weights.py:154-161 (the safetensors payload offsets come from the file headers, parsed
 * by the caller). */
int ipe_read_to_device(int files, const char* const* paths, int count, const int* file_of, const uint64_t* offsets,
                       const uint64_t* sizes, void* const* destinations, size_t staging_bytes, int threads,
                       void* stream);

/* Bytes of one rank's communication region for a tensor-parallel decode step on this device: the
 * epoch counter, two receive slots of every rank's row-parallel part, and every rank's per-CTA
 * merged LM-head records (0 for bad arguments). */
size_t ipe_decode_step_comm_bytes(int tp_world, int batch, int hidden);
size_t ipe_decode_step_workspace(int batch, int q_heads, int kv_heads, int capacity);

/* ------------------------------------------------------------------ step state */

int ipe_state_set(int64_t* state, int index, int64_t value, void* stream);
int ipe_state_add(int64_t* state, int index, int64_t delta, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* IPE_B200_H */
