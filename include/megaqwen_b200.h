/*
 * megaqwen_b200.h -- C ABI of the B200 (sm_100a) Qwen3-0.6B decode library.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t and
 * returns an int status: 0 on success, a negative MQ_ERR_* code on a host-side
 * validation failure, or a positive cudaError_t value when a CUDA call failed.
 * Nothing here takes a torch type.  Errors detected on the device (a bounded
 * wait that ran out) are reported through mq_device_status().
 *
 * The struct layouts below keep the field order of the reference's layout
 * contract (config.cuh:45-67 in Yunle-Lee/MegaQwen-A10) so that a pointer table
 * built for the reference can be passed unchanged.
 */
#ifndef MEGAQWEN_B200_H
#define MEGAQWEN_B200_H

#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Per-layer weight pointers, field order of config.cuh:45-57.  For the INT8
 * decoder the seven projection pointers point at int8 [out,in] row-major
 * codes; for the BF16 decoder at bf16 [out,in].  Norm weights are bf16. */
typedef struct LayerWeights {
    const void* input_layernorm_weight;
    const void* q_proj_weight;
    const void* k_proj_weight;
    const void* v_proj_weight;
    const void* q_norm_weight;
    const void* k_norm_weight;
    const void* o_proj_weight;
    const void* post_attn_layernorm_weight;
    const void* gate_proj_weight;
    const void* up_proj_weight;
    const void* down_proj_weight;
} LayerWeights;

/* Per-layer fp32 per-output-channel scales, field order of config.cuh:59-67. */
typedef struct ScalePointers {
    float* q_scale;
    float* k_scale;
    float* v_scale;
    float* o_scale;
    float* gate_scale;
    float* up_scale;
    float* down_scale;
} ScalePointers;

enum {
    MQ_OK = 0,
    MQ_ERR_ARG = -1,        /* null pointer, bad size or misaligned pointer */
    MQ_ERR_TOKEN = -2,      /* token id outside [0, vocab) */
    MQ_ERR_POSITION = -3,   /* position outside [0, max_seq_len) or cache_len != position+1 */
    MQ_ERR_DEVICE = -4,     /* device has too few SMs / shared memory for the kernel */
    MQ_ERR_SIZE = -5,       /* a size is larger than the entry point supports */
    MQ_ERR_DEVICE_STEP = -6 /* mq_decode_step_host: the kernel reported a device-side error */
};

/* Device-side status codes written by the decode kernel (mq_device_status). */
enum {
    MQ_DEV_OK = 0,
    MQ_DEV_TIMEOUT_EXCHANGE = 1,  /* a tagged-word exchange wait ran out */
    MQ_DEV_TIMEOUT_RING = 2,      /* a weight-ring mbarrier wait ran out */
    MQ_DEV_BAD_TOKEN = 3,         /* an input token id (device-resident) is outside [0, vocab) */
    MQ_DEV_BAD_POSITION = 4,      /* a device-resident position is outside [0, max_seq_len) */
    MQ_DEV_RANGE = 5              /* batched path: an activation outside the fp16 operand range (or not finite) */
};

/*
 * INT8 weight-only fused decode step.  Replaces launch_a10_int8_decode
 * (a10_int8_decode_kernel.cu:821-842; declared for the torch wrapper at
 * bench_int8.py:97-117) with the same argument names and order.
 *   - runs one greedy decode step at `position` (cache_len must equal
 *     position+1), writes K/V for `position` into k_cache/v_cache
 *     ([num_layers][8][max_seq_len][128] bf16), writes the final RMSNorm output
 *     to g_normalized (fp32[1024]) and the argmax token to *output_token_id
 *     (device int32).
 *   - hidden_buffer, g_activations, g_residual, g_q, g_k, g_v, g_attn_out,
 *     g_mlp_intermediate, block_max_vals and block_max_idxs are accepted for
 *     signature compatibility and not written: the kernel keeps its hand-off
 *     state in a library-owned per-device workspace.
 *   - returns a status instead of void.
 */
int launch_a10_int8_decode(
    int input_token_id, int* output_token_id,
    const void* embed_weight, const LayerWeights* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight, const float* lm_head_scale,
    const void* cos_table, const void* sin_table,
    void* k_cache, void* v_cache, void* hidden_buffer,
    void* g_activations, void* g_residual, void* g_q, void* g_k, void* g_v,
    void* g_attn_out, void* g_mlp_intermediate, void* g_normalized,
    void* block_max_vals, void* block_max_idxs,
    int num_layers, int position, int cache_len, int max_seq_len, float attn_scale,
    const ScalePointers* scales, cudaStream_t stream);

/*
 * Allocation-free INT8 decode step.  No counterpart in the reference: it is an
 * addition for callers that cannot call cudaMalloc when they decode -- a plugin
 * whose host framework owns all device memory through a pre-sized arena, or a
 * process that locks its allocator after start-up.  launch_a10_int8_decode
 * allocates its hand-off workspace on the first call on a device; this entry
 * point instead uses a workspace in a static device array of the library
 * (about 0.8 MB per GPU that loads the library, held until process exit) and
 * never calls cudaMalloc, cudaFree or any allocating routine.
 *   - Same arguments and results as launch_a10_int8_decode, without the scratch
 *     pointers the kernel does not use (hidden_buffer .. g_mlp_intermediate,
 *     block_max_vals, block_max_idxs).
 *   - Limit: num_layers <= 32 (MQ_ERR_SIZE otherwise); up to 18 attention
 *     splits per KV head, which covers every position < max_seq_len.
 *   - The first call on a device does a one-time set-up (it looks up the
 *     device address of the static array and sets the kernel's shared-memory
 *     attribute); make that first call before any stream capture.  Under CUDA's
 *     default lazy module loading that first call is also when the driver loads
 *     the library's device code and places the static array in device memory:
 *     callers whose arena claims the rest of device memory should make it during
 *     their set-up (or run with CUDA_MODULE_LOADING=EAGER).
 *   - All calls on a device share the one array, which keeps the previous
 *     call's contents (the call clears the error word itself).  Calls that
 *     overlap on the GPU -- e.g. issued on two streams without ordering --
 *     race on it: serialise them.
 *   - A device-side failure (a bounded wait that ran out) is reported only by
 *     *output_token_id == -1; the MQ_DEV_* code is not available on this path
 *     (mq_device_status reads the allocating path's workspace and allocates it
 *     on first use: do not call it here).  The next call starts clean.
 *   - The hand-off tags are 32-bit epochs advanced by (num_layers + 1) * 8 per
 *     call; the host clears the array before they wrap, counting the calls it
 *     issues.  Replays of a captured graph holding this call are not counted:
 *     keep them below 0xF0000000 / ((num_layers + 1) * 8) (about 13 million
 *     for 28 layers) between direct calls.
 */
int launch_a10_int8_decode_static(
    int input_token_id, int* output_token_id,
    const void* embed_weight, const LayerWeights* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight, const float* lm_head_scale,
    const void* cos_table, const void* sin_table, void* k_cache, void* v_cache, void* g_normalized,
    int num_layers, int position, int cache_len, int max_seq_len, float attn_scale,
    const ScalePointers* scales, cudaStream_t stream);

/* BF16 fused decode step.  Replaces launch_a10_decode
 * (a10_decode_kernel.cu:761-780): same arguments as the INT8 entry point minus
 * lm_head_scale and scales; weights are bf16. */
int launch_a10_decode(
    int input_token_id, int* output_token_id,
    const void* embed_weight, const LayerWeights* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight,
    const void* cos_table, const void* sin_table,
    void* k_cache, void* v_cache, void* hidden_buffer,
    void* g_activations, void* g_residual, void* g_q, void* g_k, void* g_v,
    void* g_attn_out, void* g_mlp_intermediate, void* g_normalized,
    void* block_max_vals, void* block_max_idxs,
    int num_layers, int position, int cache_len, int max_seq_len, float attn_scale,
    cudaStream_t stream);

/*
 * Multi-step decode with on-device token feedback (no reference counterpart:
 * the reference runs one launch plus one .item() per token,
 * bench_int8.py:193-219).  Runs `num_steps` greedy steps starting at
 * `position`; the first input token is *d_token_in (device int32) or, when
 * d_token_in is NULL, `input_token`; each later input is the previous step's
 * argmax.  Token j is written to d_tokens_out[j] (device int32).
 * weight_kind: 0 = INT8 (lm_head_scale and scales required), 1 = BF16.
 * row_pad_bytes: 0 when every weight matrix (the seven projections and the LM
 *   head) is dense row-major [out, in] as the reference stores it; 16 when each
 *   row is followed by 16 padding bytes (row stride = row bytes + 16).  The
 *   padded layout lets the kernel stream several rows with one bulk copy; the
 *   Python decoder classes repack into it once at construction.
 * d_logits (optional, may be NULL): fp32[151936] logits of the LAST step.
 * d_layer_hidden (optional, may be NULL): fp32[num_layers][1024], the bf16
 *   residual stream after each layer of the LAST step (diagnostics/parity).
 */
int mq_decode_multi(
    int weight_kind, int input_token, const int* d_token_in, int* d_tokens_out, int num_steps,
    const void* embed_weight, const LayerWeights* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight, const float* lm_head_scale,
    const ScalePointers* scales, const void* cos_table, const void* sin_table,
    void* k_cache, void* v_cache, float* g_normalized, float* d_logits, float* d_layer_hidden,
    int num_layers, int position, int max_seq_len, float attn_scale, int row_pad_bytes,
    cudaStream_t stream);

/*
 * Host-synchronous single step for the reference-facing decode_step(int) -> int
 * (bench_int8.py:193-219: one launch, then .item()).  No reference counterpart
 * as a C entry point: it exists so that the per-token host cost of that call is
 * one short C call.  The caller fills an MQStepPlan once (all pointers of the
 * decoder, which stay fixed) and passes only the token and position per step.
 *   - host_token: a pinned host int32 (cudaHostAlloc / torch pin_memory), which
 *     the kernel writes directly (mapped under unified addressing).
 *   - launches one step on `stream`, synchronises the stream and returns the
 *     token in *out_token; a device-side failure returns MQ_ERR_DEVICE_STEP
 *     (mq_device_status then has the MQ_DEV_* code).
 */
typedef struct MQStepPlan {
    int weight_kind;                 /* 0 = INT8, 1 = BF16 */
    int num_layers;
    int max_seq_len;
    int row_pad_bytes;               /* 0 or 16, as for mq_decode_multi */
    float attn_scale;
    const void* embed_weight;
    const LayerWeights* layer_weights;
    const void* final_norm_weight;
    const void* lm_head_weight;
    const float* lm_head_scale;      /* INT8 only */
    const ScalePointers* scales;     /* INT8 only */
    const void* cos_table;
    const void* sin_table;
    void* k_cache;
    void* v_cache;
    float* g_normalized;             /* optional */
    int* host_token;                 /* pinned host int32 */
} MQStepPlan;

int mq_decode_step_host(const MQStepPlan* plan, int input_token, int position, cudaStream_t stream,
                        int* out_token);

/*
 * Batched greedy decode (no reference counterpart: the
 * reference decodes one sequence).  `batch` (<= 64) independent sequences, each
 * at its own position with its own KV cache, advance num_steps tokens, sharing
 * one pass over the INT8 weights per step.  The caller owns all memory: the
 * library allocates nothing on this path.
 *   - weights (INT8, packed by mq_pack_weight_slabs): LayerWeights.q_proj_weight
 *     -> the q|k|v rows stacked (4096 x 1024) packed with block_k 256;
 *     o_proj_weight and down_proj_weight packed with block_k 256;
 *     gate_proj_weight -> gate and up pair-interleaved by 16-row tile (tile 2p =
 *     gate rows 16p..16p+15, tile 2p+1 = the same up rows; 6144 x 1024) packed
 *     with block_k 256; k/v/up pointers unused; the LM head packed with
 *     block_k 64; scales (ScalePointers, unchanged) fp32, norms and embedding bf16;
 *   - k_cache / v_cache: bf16 [batch][num_layers][8][max_seq_len][128]
 *     (batch * num_layers * 8 * max_seq_len below 2^31 rows, else MQ_ERR_SIZE:
 *     the kernel reads them through 2-D TMA tensor maps with 32-bit row
 *     coordinates);
 *   - tokens: device int32 [batch]: read as this step's inputs, overwritten
 *     with the argmax outputs (so repeated steps feed back on the device);
 *   - positions: device int32 [batch]: position of each sequence's input token
 *     (cache_len = position + 1); incremented by one per step;
 *   - workspace: device buffer of mq_batch_workspace_bytes(batch) bytes,
 *     16-byte aligned, zero-filled before its first use;
 *   - logits (optional): fp32 [batch][151936] of the last step;
 *   - max_seq_len <= 32768.
 * A device-side failure leaves tokens at -1; mq_batch_status() reads the code.
 * The GEMMs run on the tcgen05 tensor cores with fp16 operands: INT8 weights
 * are dequantised exactly to fp16 in shared memory; activations enter as fp16
 * of x * 2^-s (s = 8 for RMSNorm inputs, 4 otherwise; 11 significant bits);
 * fp32 accumulation.  A value beyond the fp16 range stops the step with
 * MQ_DEV_RANGE.
 */
typedef struct MQBatchArgs {
    const void* embed_weight;
    const LayerWeights* layer_weights;   /* device array [num_layers] */
    const ScalePointers* scales;         /* device array [num_layers] */
    const void* final_norm_weight;
    const void* lm_head_weight;
    const float* lm_head_scale;
    const void* cos_table;
    const void* sin_table;
    void* k_cache;
    void* v_cache;
    int* tokens;
    int* positions;
    void* workspace;
    size_t workspace_bytes;
    float* logits;
    unsigned long long* trace;           /* optional diagnostics: [num_ctas][8*(num_layers+1)] %globaltimer
                                            stamps, slot layer*8+phase (1 QKV .. 6 down done), 8L+6/7 LM */
    unsigned long long wait_budget_ns;   /* 0: default (2 s) */
    int batch;
    int num_layers;
    int max_seq_len;
    float attn_scale;
    int prefill;                         /* 0: independent sequences.  1: chunked prefill -- the rows are
                                            consecutive tokens of ONE sequence at consecutive positions,
                                            all sharing the cache of row 0 ([num_layers][8][max_seq][128]);
                                            every row's K/V is written before attention, which reads
                                            positions [0, position] from the cache; num_steps must be 1 */
    int vocab_shards, vocab_shard;       /* vocab-sharded LM head (G ranks decoding the same sequences):
                                            this call scores only shard vocab_shard of vocab_shards
                                            (contiguous 16-row tiles) and writes keys_out instead of tokens;
                                            0 / 0: whole vocabulary */
    long long* keys_out;                 /* [batch] packed argmax keys ((order(logit) << 32 | ~row) with the
                                            sign bit flipped): the max over the shards (an int64 max
                                            all-reduce) is the global argmax, lowest row on ties; the
                                            token is ~key & 0xffffffff.  Requires num_steps == 1 */
} MQBatchArgs;

int mq_batch_workspace_bytes(int batch, size_t* bytes);
int mq_batch_decode(const MQBatchArgs* args, int num_steps, cudaStream_t stream);
/* Device-side status of a batched workspace (synchronous copy): MQ_DEV_* code. */
int mq_batch_status(const void* workspace, int* code, int* info);

/*
 * Packs an INT8 weight matrix [rows][K] (row stride src_row_stride bytes,
 * a multiple of 8) for the batched path: 16-row x 64-column blocks of 1 KB,
 * block (tile, kb) at byte ((tile * K/64) + kb) * 1024, inside ordered
 * [8-column group][16 rows][8 bytes].  rows % 16 == 0, K % 64 == 0; dst holds
 * rows * K bytes, 16-byte aligned.  Asynchronous on `stream`.
 */
int mq_pack_weight_tiles(const int8_t* src, int64_t rows, int K, int64_t src_row_stride, int8_t* dst,
                         cudaStream_t stream);
/* Slab-major blocks of block_k (64 or 256) columns: block (kb, tile) at byte
 * ((kb * rows/16) + tile) * 16 * block_k, inside [8-column group][16 rows][8 bytes],
 * so the consecutive row tiles of one slab are contiguous and a CTA's rows of a
 * slab are one copy.  The batched path uses block_k = 256 for the projections
 * and 64 for the LM head. */
int mq_pack_weight_slabs(const int8_t* src, int64_t rows, int K, int64_t src_row_stride, int block_k,
                         int8_t* dst, cudaStream_t stream);

/*
 * The batched path's tensor-core GEMM on its own:
 * y[t][m] = scale[m] * sum_k W[m][k] * x[t][k] for t < B <= 64, W tile-packed
 * [M][K] INT8 (M % 16 == 0, K in {1024, 2048, 3072}), x fp32 [B][K], y fp32
 * [B][M] (x enters the tensor cores as fp16, |x| <= 65504); workspace of
 * mq_batch_matmul_workspace_bytes(K) bytes, 16-byte aligned.  Asynchronous on
 * `stream`; mq_batch_status(workspace) reads a device-side timeout or range
 * error.
 */
int mq_batch_matmul_workspace_bytes(int K, size_t* bytes);
int mq_batch_matmul(const int8_t* w_tiles, const float* scale, const float* x, float* y, int M, int K, int B,
                    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * Per-output-channel symmetric INT8 quantizer.  Same arithmetic as
 * quantize_per_channel (bench_int8.py:19-24): absmax in bf16,
 * scale = fp32(bf16(absmax/127)) clamped to >= 1e-12,
 * q = clamp(round_half_even(fp32(w)/scale), -128, 127).
 * w: bf16 [M,K] row-major; q: int8 [M,K]; scale: fp32 [M].
 */
int mq_quantize_per_channel(const void* w_bf16, int64_t M, int64_t K,
                            int8_t* q_out, float* scale_out, cudaStream_t stream);

/*
 * Standalone weight-only matvec, y[m] = scale[m] * sum_k W[m,k] * x[k]
 * (the per-projection math of a10_int8_decode_kernel.cu:87-136 and
 * int8_gemv, int8_decoder.py:100-115).  weight_kind 0 = int8 W with fp32
 * scale, 1 = bf16 W (scale ignored, may be NULL).  x, y fp32 on the device.
 * K must be one of 1024, 2048, 3072.
 */
int mq_matvec(int weight_kind, const void* W, const float* scale, const float* x,
              float* y, int M, int K, cudaStream_t stream);

/* Reads (and with clear != 0, clears) the device-side status of this device's
 * decode workspace.  Synchronises the device.  *code gets an MQ_DEV_* value,
 * *info the kernel's location code for it. */
int mq_device_status(int* code, int* info, int clear);

/* Sets the bounded-wait budget (nanoseconds) that every spin in the decode
 * kernel uses before it gives up with MQ_DEV_TIMEOUT_*.  Default 2e9. */
int mq_set_wait_budget_ns(uint64_t ns);

/* Test hook: when nonzero, the next decode launch's CTA `cta` skips writing
 * its share of the QKV exchange, so every consumer of it runs into the
 * bounded wait and reports MQ_DEV_TIMEOUT_EXCHANGE.  Cleared after one launch. */
int mq_inject_skip_publish(int enable, int cta);

/* Tracing: when dev_buf is non-NULL, every later decode launch writes
 * %globaltimer stamps (ns) into dev_buf[cta * slots_per_cta + slot], slot =
 * layer * 10 + event (events: 0 layer input ready, 1 QKV published, 2 attention
 * published, 3 attention gathered, 4 O published, 5 post-norm done, 6 gate/up
 * published, 7 MLP gathered, 8 down published; slots num_layers*10 + 0/1/2/3:
 * final hidden gathered / LM head done / CTA entered the kernel / CTA done).
 * NULL disables.  No reference counterpart
 * (the reference has no tracing). */
int mq_set_trace(unsigned long long* dev_buf, int slots_per_cta);

/* Number of CTAs (one per SM) and dynamic shared memory the decode kernel uses. */
int mq_kernel_info(int* num_ctas, int* smem_bytes, int* threads);

/* Diagnostics of the current device (no reference counterpart):
 * binary_version: the decode kernel's cudaFuncAttributes::binaryVersion
 *   (100 = built for sm_100a and loaded as such);
 * workspace_allocated: 1 if the allocating entry points have created their
 *   per-device workspace on this device, else 0.  Allocates nothing. */
int mq_library_info(int* binary_version, int* workspace_allocated);

#ifdef __cplusplus
}
#endif
#endif
