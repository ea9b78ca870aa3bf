// decode.cuh -- data structures of the persistent decode kernel.
#pragma once
#include "common.cuh"

namespace mq {

constexpr int PART_WORDS = 2 * HD + 4;  // acc[2][128], m[2], l[2] per attention split
constexpr int TAGS_PER_LAYER = 8;

// Library-owned per-device workspace.  Hand-off buffers are double-buffered by
// layer parity; every word carries the epoch tag of the exchange that wrote it.
struct Workspace {
    uint32_t epoch;                 // tag base of the next launch
    uint32_t exit_ctr;              // CTAs that finished the current launch
    unsigned long long argmax;      // packed (order_key(logit) << 32 | ~row)
    int err_code;                   // first MQ_DEV_* error of any launch since cleared
    int err_info;                   // location code of that error
    int pad_[10];
    uint64_t xh[2][HIDDEN];         // residual stream h (bf16 payload), input of layer l
    uint64_t xqkv[2][QKV_ROWS];     // raw q|k|v projections (fp32)
    uint64_t xattn[2][QSZ];         // attention output per q head (fp32)
    uint64_t xact[2][HIDDEN];       // h + O-proj (fp32)
    uint64_t xmlp[2][INTER];        // silu(gate)*up (fp32)
    uint64_t xpart[2][NKVH * MAX_SPLITS * PART_WORDS];  // split-K attention partials
};

struct DecodeParams {
    const void* embed;
    const LayerWeights* layers;     // device array [L]
    const ScalePointers* scales;    // device array [L] (INT8 only)
    const void* final_norm;
    const void* lm_w;
    const float* lm_scale;          // INT8 only
    const __nv_bfloat16* cos_t;
    const __nv_bfloat16* sin_t;
    __nv_bfloat16* kc;
    __nv_bfloat16* vc;
    float* g_normalized;            // optional fp32[1024]
    float* logits;                  // optional fp32[VOCAB]
    float* layer_hidden;            // optional fp32[L][1024]
    const int* token_in_dev;        // optional; else token_in
    int* token_out;                 // device int32
    Workspace* ws;
    unsigned long long budget_ns;
    int token_in;
    int L;
    int position;                   // cache_len = position + 1
    int max_seq;
    int splits;                     // attention splits per KV head
    float attn_scale;
    int skip_cta;                   // test hook: CTA that skips its layer-0 QKV publish (-1: none)
    unsigned long long* trace;      // optional [gridDim.x][trace_slots] globaltimer stamps
    int trace_slots;
    int row_pad;                    // 0: weight rows dense (reference layout); ROW_SKEW: rows padded to rb + ROW_SKEW
    int kv_pf_pos;                  // cached positions of the next layer's KV each attention split prefetches into L2
};

// Trace slots: per layer l, stamps at l * TRACE_PER_LAYER + event.
enum { TR_START = 0, TR_QKV = 1, TR_ATTN = 2, TR_OIN = 3, TR_O = 4, TR_NORM2 = 5, TR_GU = 6, TR_MLPIN = 7,
       TR_DOWN = 8, TRACE_PER_LAYER = 10 };

// Shared-memory layout (dynamic).
static_assert(NCW <= 12, "attention merge uses x[NCW][2][HD] as scratch");
static_assert(NCT >= 2 * HD, "attention merge: one consumer thread per (GQA head, dim)");
static_assert(KV_CHUNK_POS <= 32, "");
static_assert(STAGE_BYTES >= 2 * INTER + ROW_SKEW && STAGE_BYTES >= 2 * (2 * HIDDEN + ROW_SKEW),
              "a stage must hold one bf16 down row and one bf16 gate+up pair");
static_assert(STAGE_BYTES >= 16 * (HIDDEN + ROW_SKEW), "16 int8 rows of 1024 per stage (one mma tile)");
struct Smem {
    uint8_t ring[NSTAGE][STAGE_BYTES];
    uint64_t full[NSTAGE];
    uint64_t empty[NSTAGE];
    float h[HIDDEN];         // residual stream (fp32 copy of bf16 h)
    float act[HIDDEN];       // h + O (residual of the MLP half)
    float x[INTER];          // current matvec activation (normalized / attn / mlp)
    float red[NCW];
    float red2[NCW];
    float limb_inv;
    alignas(16) int limb[4][INTER / 4];  // activation limbs of the current matvec phase; row 3 stays zero
    float raw[4 * HD];       // raw q0 q1 k v of this CTA's KV head
    alignas(16) float q[2][HD];
    float m[2], l[2], corr[2];
    float sc[2][32];         // per-warp softmax state during the attention merge
    float pe[2][32];
    float ew[2][32];         // merge weights exp(m_w - M_h)
    float lw_[2][32];        // l_w * ew
    float mx[2];
    alignas(16) uint16_t kvcur[2][HD];   // current-position K and V, bf16
    unsigned long long best[NCW];
    const void* lw[MAX_LAYERS][11];      // LayerWeights of every layer
    const float* ls[MAX_LAYERS][7];      // ScalePointers of every layer
    float scl[MAX_LAYERS * SCL_STRIDE];  // this CTA's per-row scales of every layer
    float lm_scl[LM_MAXR + 1];           // this CTA's LM-head row scales
    int abort_flag;
};

}  // namespace mq
