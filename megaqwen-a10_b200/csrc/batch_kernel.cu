// batch_kernel.cu -- batched greedy decode of Qwen3-0.6B on B200 (sm_100a):
// B <= 64 independent sequences (each at its own position, with its own KV
// cache) advance one token per launch, sharing one pass over the INT8 weights.
//
// Per layer six phases separated by bounded grid barriers (a batched step is
// KV-bound, milliseconds, so ~1.2 us per barrier is affordable and all data
// moves through plain global buffers):
//   QKV   GEMM on the 5th-generation tensor cores (tcgen05.mma, accumulator in
//         TMEM) -> qkv[b][4096] fp32
//   ATTN  one equal range of (sequence, KV head, position) per warp: QK-RMSNorm
//         + RoPE at the sequence's own position, K/V write, flash-decode over
//         the cached positions (KV chunks bulk-copied into the warp's shared
//         buffer) -> partials (m, l, acc)
//   MERGE one warp per (sequence, q head): merges the splits -> O operand
//   O     GEMM + residual -> act fp32, GU operand
//   GU    gate and up GEMM, SiLU(gate)*up -> DOWN operand
//   DOWN  GEMM + residual -> h (rounded to bf16, as between layers of the
//         batch-1 kernel), next QKV (or LM-head) operand
// then the LM-head GEMM with a per-sequence packed argmax.  Prefill mode
// (rows = consecutive tokens of one sequence sharing its cache) adds a K/V
// write sub-phase and a barrier before attention; vocab-sharded mode scores
// one slice of the vocabulary and emits packed argmax keys.
//
// GEMM shape.  D[128 x N] = X[128 x K] * W[N x K]^T: rows 0..63 of X are the
// 64 sequences' activations as fp16 of x * 2^-s (rows 64..127 are don't-care
// and their accumulator rows are never read), N = this CTA's weight rows
// (16-row tiles, N <= 256), K streamed in slabs through a ring of shared-memory
// slots fed by bulk copies:
//   * the activation operand lives in global memory already in the tensor
//     core's K-major no-swizzle layout (8-wide k columns of [64 rows][16 B]),
//     written by the producing phase's epilogue, so a slab is ONE bulk copy;
//   * the INT8 weights are packed once at load time slab-major (blocks of 16
//     rows x 256 k for the projections, 16 x 64 for the LM head, [8-k
//     column][row][8 B] inside), so this CTA's rows of a slab are one bulk
//     copy; the CTA dequantises them to fp16 (exact) in shared memory in the
//     same K-major layout and two threads issue the tcgen05.mma instructions;
//   * the per-row weight scale, 2^s and, for RMSNorm inputs, the per-sequence
//     1/rms multiply the fp32 accumulator in the epilogue, read back from TMEM
//     with tcgen05.ld.
// RMSNorm inputs are written as h*w (norm weight applied, 1/rms not) together
// with per-16-row partial sums of squares; the consumer reduces the 64 partials
// in a fixed order, so results are deterministic.
#include "common.cuh"
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdlib.h>

namespace mq {
namespace batch {

constexpr int BMAX = 64;                 // sequences per launch
constexpr int NW = 12;                   // warps per CTA
constexpr int NT = NW * 32;
constexpr int MROWS = 128;               // MMA M (rows 0..63: the sequences; 64..127 unused)
constexpr int XCOL = BMAX * 16;          // bytes of one 8-wide k column of the activation operand
constexpr int HROWS = BMAX / 2;          // token-half operands (O, down): 32 rows
constexpr int HXCOL = HROWS * 16;        // bytes of one 8-wide k column of a token-half operand
// Activation operands are stored as fp16 of x * 2^-s (exact power-of-two
// pre-scale, undone in the epilogue): s = 8 for RMSNorm inputs (h * w, which
// carry the residual stream's magnitude), 4 for attention and MLP outputs.
// |x * 2^-s| must stay below 65504; a larger (or non-finite) value stops the
// step with MQ_DEV_RANGE instead of being rounded silently.
constexpr float XS_NORM = 1.0f / 256.0f;
constexpr float XS_ACT = 1.0f / 16.0f;
constexpr int TROWS = 16;                // weight rows per packed tile
constexpr int KBLK = 64;                 // k per packed 1 KB block
#ifndef MQB_NR
#define MQB_NR 8
#endif
constexpr int NR = MQB_NR;               // ring slots at most (their size depends on the GEMM)
constexpr int RING = 192 * 1024;         // ring bytes
#ifndef MQB_NMMA
#define MQB_NMMA 2
#endif
constexpr int NMMA = MQB_NMMA;           // MMA-issuing threads (warps 1 .. NMMA), one accumulator each
constexpr int NDQ = NW - 1 - NMMA;       // dequantising warps of the GEMM pipeline
constexpr int ACC_COLS = 256;            // fp32 accumulator columns (N <= 256)
constexpr int TMEM_COLS = NMMA == 1 ? 256 : 512;   // one accumulator per MMA issuer
constexpr int MAX_TILES_PASS = ACC_COLS / TROWS;
constexpr int HT = HIDDEN / TROWS;       // 64 row tiles of the hidden dimension (sum-of-squares partials)
constexpr int ACH = 16;                  // positions per KV chunk (one m16n8k16 tile of positions)
#ifndef MQB_NBUF
#define MQB_NBUF 2
#endif
#ifndef MQB_NAW
#define MQB_NAW 12
#endif
constexpr int NBUF = MQB_NBUF;           // KV chunk buffers per attention warp
constexpr int NAW = MQB_NAW;             // attention warps per CTA
static_assert(NAW * NBUF * 2 * ACH * HD * 2 <= 192 * 1024, "attention buffers exceed the ring");
constexpr int MAX_SPLITS_B = 130;        // partials per (sequence, KV head): 32768 / 256 + 2
constexpr int PARTW = 2 * HD + 4;        // acc[2][128], m[2], l[2]

// Ring slot contents for slab width KS and N weight rows: activation slab
// (128 x KS bf16), dequantised weight slab (N x KS bf16), raw weight slab (N x KS int8).
template <int KS>
struct SlabGeom {
    static constexpr int A_BYTES = BMAX * KS * 2;
    __device__ static int slot_bytes(int n) { return (A_BYTES + 3 * n * KS + 1023) & ~1023; }
};
static_assert(3 * (BMAX * 64 * 2 + 3 * 256 * 64) <= RING, "ring too small for three N = 256 slabs");
static_assert(2 * (BMAX * 128 * 2 + 3 * 80 * 128) <= RING, "ring too small for two N = 80 slabs");

struct Params {
    // K / V caches as 2-D tensors [rows = B * L * 8 * max_seq][128] bf16, box 16 rows x 64 dims, 128-byte
    // swizzle: the attention warps fetch 16-position chunks with TMA so that ldmatrix reads them conflict-free
    CUtensorMap tm_k, tm_v;
    // weights: INT8 matrices packed slab-major (mq_pack_weight_slabs; see MQBatchArgs)
    const __nv_bfloat16* embed;
    const LayerWeights* layers;
    const ScalePointers* scales;
    const __nv_bfloat16* final_norm;
    const int8_t* lm_w;
    const float* lm_scale;
    const __nv_bfloat16* cos_t;
    const __nv_bfloat16* sin_t;
    // per-sequence state
    __nv_bfloat16* kc;          // [B][L][8][max_seq][128]
    __nv_bfloat16* vc;
    const int* tokens_in;       // [B]
    int* tokens_out;            // [B]
    int* positions;             // [B] position of the token being decoded (cache_len = pos + 1); advanced by 1 per step
    // workspace
    float* h;                   // [B][1024] residual stream
    float* act;                 // [B][1024] residual after attention
    float* qkv;                 // [B][4096]
    uint8_t* xa_qkv;            // GEMM operands (K = 1024, 2048, 1024, 3072); xa_qkv also feeds the LM head
    uint8_t* xa_o;
    uint8_t* xa_gu;
    uint8_t* xa_dn;
    float* ss_a;                // [HT][BMAX] partial sums of squares of h (QKV / LM-head RMSNorm)
    float* ss_b;                // [HT][BMAX] of act (post-attention RMSNorm)
    float* part;                // [B][8][MAX_SPLITS_B][PARTW]
    unsigned long long* best;   // [B]
    unsigned int* ctl;          // [0] barrier counter, [1] exit counter, [2] error code, [3] error info
    float* logits;              // optional [B][VOCAB]
    unsigned long long* trace;  // optional [gridDim.x][8 * (L + 1)] globaltimer stamps
    unsigned long long budget_ns;
    int B, L, max_seq;
    float attn_scale;
    int prefill;                // rows = consecutive tokens of ONE sequence sharing row 0's KV cache
    int lm_tile0, lm_tiles;     // LM-head vocab shard: 16-row tiles [lm_tile0, lm_tile0 + lm_tiles)
    long long* keys_out;        // vocab-sharded mode: per-sequence packed argmax keys (sign-flipped) instead of tokens
};

// ---------------------------------------------------------------------------
// Shared memory (phases use disjoint views of one buffer)
// ---------------------------------------------------------------------------
struct AttnSmem {
    alignas(1024) uint8_t kv[NAW][NBUF][2 * ACH * HD * 2];   // per warp: NBUF chunks of ACH positions (K then V)
    alignas(16) float q[NW][2][HD];
};
struct Smem {
    union {
        alignas(1024) uint8_t ring[RING];         // GEMM slab slots; after the last MMA, the fp32 epilogue tile
        AttnSmem a;
    };
    uint64_t full[NR];       // slab copies landed
    uint64_t mdone[NR];      // MMAs reading the slot completed (tcgen05.commit)
    uint64_t deq[NR];        // slot's weights dequantised (one arrival per dequantising warp)
    uint64_t abar[NAW][NBUF]; // per-warp KV chunk copies
    unsigned long long tokbest[BMAX];
    float rstd[BMAX];        // per-sequence 1/rms of the GEMM input being consumed
    int seqoff[BMAX + 1];    // attention work split: flattened start of each sequence
    int segq;                // and the range length per warp
    uint32_t tmem_base;
    int abort_flag;
};

static_assert(sizeof(Smem) + 1024 <= 227 * 1024, "shared memory (plus the alignment KB) exceeds 227 KB");

struct Ctx {
    Smem* sm;
    unsigned int* ctl;
    unsigned long long budget;
    uint32_t tmem;
    unsigned int barriers;   // grid barriers passed in this launch
    uint32_t upar;           // bit i: parity of the next use of ring slot i (mbarrier phase)
    uint32_t pend;           // ring slots with copies issued and not known complete (producer)
    uint32_t ppar;           // bit i: parity of the last copy issued into slot i
    int mma_slot;            // slot of the last commit nobody waited for (-1: none)
    int half;                // -1: the operand holds all 64 sequences; 0 / 1: token-half operand (32 rows)
    uint32_t mma_par;
};

__device__ __forceinline__ bool aborted(Ctx& c) {
    if (*(volatile int*)&c.sm->abort_flag) return true;
    if (ld_relaxed32(&c.ctl[2]) != 0) { *(volatile int*)&c.sm->abort_flag = 1; return true; }
    return false;
}
__device__ __noinline__ void fail(Ctx& c, int code, int info) {
    if (atomicCAS(&c.ctl[2], 0u, (unsigned)code) == 0u) atomicExch(&c.ctl[3], (unsigned)info);
    *(volatile int*)&c.sm->abort_flag = 1;
}

__device__ __forceinline__ void stamp(const Params& P, int slot) {
    if (P.trace && threadIdx.x == 0) P.trace[(size_t)blockIdx.x * 8 * (P.L + 1) + slot] = globaltimer();
}

// Bounded grid barrier (release/acquire on a monotone counter reset per launch).
// Returns false when any CTA has failed; the caller then leaves the step.
__device__ bool grid_barrier(Ctx& c, int where) {
    // Global and shared bytes written through the generic proxy in this phase
    // are read (or overwritten) by bulk copies -- the async proxy -- in the next.
    asm volatile("fence.proxy.async;" ::: "memory");
    __syncthreads();
    bool ok = !*(volatile int*)&c.sm->abort_flag;
    if (threadIdx.x == 0) {
        ++c.barriers;
        const unsigned target = c.barriers * gridDim.x;
        __threadfence();
        atomicAdd(&c.ctl[0], 1u);
        unsigned long long t0 = globaltimer();
        for (uint32_t it = 0;; ++it) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(&c.ctl[0]) : "memory");
            if ((int)(v - target) >= 0) break;
            if ((it & 63) == 63) {
                if (ld_relaxed32(&c.ctl[2]) != 0) { c.sm->abort_flag = 1; break; }
                if (globaltimer() - t0 > c.budget) { fail(c, MQ_DEV_TIMEOUT_EXCHANGE, where); break; }
            }
        }
    } else {
        ++c.barriers;
    }
    __syncthreads();
    return ok && !*(volatile int*)&c.sm->abort_flag;
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Bounded mbarrier wait; gives up early when the step is aborted.
__device__ __forceinline__ bool mbar_wait_b(Ctx& c, uint64_t* bar, uint32_t parity, int where) {
    if (mbar_test(bar, parity)) return true;
    unsigned long long t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_test(bar, parity)) return true;
        if ((it & 63) == 0) {
            if (aborted(c)) return false;
            if (globaltimer() - t0 > c.budget) { fail(c, MQ_DEV_TIMEOUT_RING, where); return false; }
        }
    }
}
// Bounded wait used while leaving after a failure: ignores the abort flag.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity, unsigned long long budget) {
    const unsigned long long t0 = globaltimer();
    while (!mbar_test(bar, parity))
        if (globaltimer() - t0 > budget) return;
}

// ---------------------------------------------------------------------------
// tcgen05 pieces
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, no swizzle: 8 x 16 B core matrices;
// lbo = byte distance of core matrices adjacent in K, sbo = of core matrices
// adjacent in M/N (8-row groups); descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor, kind::f16: fp16 A and B (both K-major), fp32 D, M = 128, N.
__device__ __forceinline__ uint32_t idesc_f16(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(MROWS >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accum)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 32 lanes x 8 consecutive fp32 columns (this warp's lane quadrant); waits for the load.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// Four signed bytes -> four fp16 (exact).  Byte b is placed as the low mantissa
// byte of an fp16 whose exponent makes it 1024 + (b + 128) (the ulp at 1024 is
// 1), then 1152 is subtracted: two byte permutes and two packed subtractions.
__device__ __forceinline__ void i8x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t x = w ^ 0x80808080u;   // b + 128 as an unsigned byte
    uint32_t a, b;
    asm("prmt.b32 %0, %1, %2, 0x4140;" : "=r"(a) : "r"(x), "r"(0x64646464u));   // {0x64, x1, 0x64, x0}
    asm("prmt.b32 %0, %1, %2, 0x4342;" : "=r"(b) : "r"(x), "r"(0x64646464u));   // {0x64, x3, 0x64, x2}
    const __half2 bias = __float2half2_rn(1152.0f);
    const __half2 ra = __hsub2(*reinterpret_cast<const __half2*>(&a), bias);
    const __half2 rb = __hsub2(*reinterpret_cast<const __half2*>(&b), bias);
    lo = *reinterpret_cast<const uint32_t*>(&ra);
    hi = *reinterpret_cast<const uint32_t*>(&rb);
}
// Two signed bytes -> two fp16 (exact: |v| <= 128).
__device__ __forceinline__ uint32_t i8x2_to_f16x2(uint32_t v) {
    const __half2 h = __halves2half2(__int2half_rn((int)(int8_t)(v & 0xffu)), __int2half_rn((int)(int8_t)((v >> 8) & 0xffu)));
    return *reinterpret_cast<const uint32_t*>(&h);
}

// x[0..7] * sc as eight fp16 (one 16-byte row of an 8-wide k column); false if a
// value is outside the fp16 range (or not finite).
__device__ __forceinline__ bool pack_x8(const float* x, float sc, uint4& out) {
    uint32_t w[4];
    bool ok = true;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float a = x[2 * i] * sc, b = x[2 * i + 1] * sc;
        ok &= fabsf(a) <= 65504.f && fabsf(b) <= 65504.f;
        const __half2 h = __floats2half2_rn(a, b);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    out = make_uint4(w[0], w[1], w[2], w[3]);
    return ok;
}
// Writes x[0..7] * sc (k0 .. k0 + 7 of sequence t, k0 % 8 == 0) into an
// activation operand as fp16 (row t of the 8-wide k column).
__device__ __forceinline__ bool put_x8(uint8_t* xa, int t, int k0, const float* x, float sc) {
    uint4 v;
    const bool ok = pack_x8(x, sc, v);
    *reinterpret_cast<uint4*>(xa + (size_t)(k0 >> 3) * XCOL + t * 16) = v;
    return ok;
}
// The same into a token-half operand of K columns: [half][k column][32 rows][16 B].
__device__ __forceinline__ bool put_x8h(uint8_t* xa, int K, int t, int k0, const float* x, float sc) {
    uint4 v;
    const bool ok = pack_x8(x, sc, v);
    *reinterpret_cast<uint4*>(xa + (size_t)(t / HROWS) * (K / 8) * HXCOL + (size_t)(k0 >> 3) * HXCOL +
                              (t % HROWS) * 16) = v;
    return ok;
}
__device__ __noinline__ void range_fail(unsigned* ctl, int where) {
    if (atomicCAS(&ctl[2], 0u, (unsigned)MQ_DEV_RANGE) == 0u) atomicExch(&ctl[3], (unsigned)where);
}

// Loads 16 fp32 values [k0, k0 + 16) of a row written by other CTAs (L2).
__device__ __forceinline__ void load16(const float* row, int k0, float (&v)[16]) {
    const float4* r = reinterpret_cast<const float4*>(row + k0);
    float4 q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = __ldcg(r + i);
#pragma unroll
    for (int i = 0; i < 4; ++i) { v[4 * i] = q[i].x; v[4 * i + 1] = q[i].y; v[4 * i + 2] = q[i].z; v[4 * i + 3] = q[i].w; }
}
__device__ __forceinline__ void store16(float* row, int k0, const float (&v)[16]) {
    float4* r = reinterpret_cast<float4*>(row + k0);
#pragma unroll
    for (int i = 0; i < 4; ++i) r[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}
__device__ __forceinline__ void load16_bf16(const __nv_bfloat16* row, int k0, float (&v)[16]) {
    const uint4* r = reinterpret_cast<const uint4*>(row + k0);
    const uint4 a = __ldg(r), b = __ldg(r + 1);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) { v[2 * i] = bf16_bits_to_f32(w[i] & 0xffffu); v[2 * i + 1] = bf16_bits_to_f32(w[i] >> 16); }
}
// Accumulator row of sequence t, columns [col, col + 16) of the epilogue tile, times inv.
__device__ __forceinline__ void erow16(const float* E, int ldE, int t, int col, float inv, float (&v)[16]) {
    const float4* a = reinterpret_cast<const float4*>(E + (size_t)t * ldE + col);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 x = a[i];
        v[4 * i] = x.x * inv; v[4 * i + 1] = x.y * inv; v[4 * i + 2] = x.z * inv; v[4 * i + 3] = x.w * inv;
    }
}
// 1/rms of each sequence from the 64 per-tile partial sums (fixed order).
// Run by the dequantising warps: the producer and MMA warps start the
// GEMM pipeline meanwhile; the result is read after the GEMM's final barrier.
__device__ __forceinline__ void compute_rstd(Smem* sm, const float* ss, int B) {
    for (int t = (int)threadIdx.x - 32 * (NMMA + 1); t < B; t += NT - 32 * (NMMA + 1)) {
        if (t < 0) break;
        float s = 0.f;
#pragma unroll 16
        for (int j = 0; j < HT; ++j) s += __ldcg(ss + j * BMAX + t);
        sm->rstd[t] = rsqrtf(s / (float)HIDDEN + RMS_EPS);
    }
}

// ---------------------------------------------------------------------------
// The GEMM of one CTA: D[128 x 16 nt] = X * W^T over K, tiles given by
// tile_ptr(j) (packed tile base, j < nt).  Warp-specialised pipeline over the
// K slabs, linked by mbarriers (no CTA-wide barrier per slab):
//   warp 0 lane 0    producer: bulk copies of slab s into slot s % nr once the
//                    MMAs of slab s - nr have completed (mdone);
//   warps 1..NMMA    lane 0: MMA issuer k takes slabs k, k + NMMA, ... into its
//                    own TMEM accumulator (summed in the epilogue): waits for
//                    the slot's copies (full) and dequantised weights (deq),
//                    issues the tcgen05.mma instructions, commits to mdone.
//                    One issuer alone could not keep up with the slab rate;
//   other warps      dequantisers: wait for the copies (full), INT8 -> fp16
//                    into the slot's operand area, one arrival per warp on deq.
// On success the fp32 accumulator is left in shared memory as E[rows][ldE]
// (aliasing the ring) and all threads have passed a barrier; the caller runs
// its epilogue on E and must fence_proxy_async() + __syncthreads() before the
// ring is used again.
// ---------------------------------------------------------------------------
template <int KS, class TilePtr>
__device__ bool tc_gemm(Ctx& c, const uint8_t* xa, int K, int nt, TilePtr tile_ptr, const float*& E, int& ldE,
                        const int8_t* slab_base = nullptr, int slab_ntm = 0, int slab_g0 = 0) {
    using G = SlabGeom<KS>;
    Smem* sm = c.sm;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int N = nt * TROWS, S = K / KS;
    const int BB = 2 * N * KS, BR = N * KS;
    // activation operand: 64 rows, or (token-half operands, stored [half][k column][32 rows][16 B]) 32 rows
    const int XC = c.half >= 0 ? HXCOL : XCOL;
    const int AB = XC / 16 * KS * 2;
    const uint8_t* xs = xa + (c.half >= 0 ? (size_t)c.half * (K / 8) * HXCOL : 0);
    const uint32_t tx = (uint32_t)(AB + BR);
    const int SB = (AB + 3 * N * KS + 1023) & ~1023;
    const int nr = min(NR, RING / SB);
    if (nr < NMMA) {   // the MMA issuers alternate slots: each needs one (static_asserts cover the shapes used)
        if (threadIdx.x == 0) fail(c, MQ_DEV_RANGE, 299);
        return false;
    }
    const uint32_t par0 = c.upar;   // parity of the next use of each slot
    // parity of the mbarrier phases of slab s (its slot's (s / nr)-th use in this GEMM)
    auto par = [&](int s) { return ((par0 >> (s % nr)) ^ (uint32_t)(s / nr)) & 1u; };
    bool ok = true;
    if (warp == 0) {
        if (lane == 0) {
            for (int s = 0; s < S; ++s) {
                const int slot = s % nr;
                if (s >= nr) {   // the slot's previous MMAs must have finished reading it
                    ok = mbar_wait_b(c, &sm->mdone[slot], par(s - nr), 220 + slot);
                    if (!ok) break;
                }
                uint8_t* base = sm->ring + slot * SB;
                mbar_arrive_expect_tx(&sm->full[slot], tx);
                bulk_g2s(base, xs + (size_t)s * AB, AB, &sm->full[slot]);
                if (slab_ntm > 0)   // slab-major packing (block width KS): the nt tiles of this slab are contiguous
                    bulk_g2s(base + AB + BB, slab_base + ((size_t)s * slab_ntm + slab_g0) * (TROWS * KS),
                             nt * TROWS * KS, &sm->full[slot]);
                else
                    for (int j = 0; j < nt; ++j)
                        bulk_g2s(base + AB + BB + j * TROWS * KS, tile_ptr(j) + (size_t)s * TROWS * KS,
                                 TROWS * KS, &sm->full[slot]);
                c.pend |= 1u << slot;
                c.ppar = (c.ppar & ~(1u << slot)) | (par(s) << slot);
            }
        }
    } else if (warp <= NMMA) {
        // MMA issuer k = warp - 1 takes slabs s = k, k + NMMA, ... into accumulator k
        if (lane == 0) {
            const int k = warp - 1;
            const uint32_t idesc = idesc_f16(N);
            const uint32_t acc = c.tmem + (uint32_t)(k * ACC_COLS);
            for (int s = k; s < S; s += NMMA) {
                const int slot = s % nr;
                ok = mbar_wait_b(c, &sm->full[slot], par(s), 250 + slot) &&   // copies landed
                     mbar_wait_b(c, &sm->deq[slot], par(s), 240 + slot);     // weights dequantised
                if (!ok) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(sm->ring + slot * SB), b0 = a0 + AB;
#pragma unroll
                for (int i = 0; i < KS / 16; ++i)
                    umma_f16(acc, sdesc(a0 + i * 2 * XC, XC, 128), sdesc(b0 + i * 2 * N * 16, N * 16, 128), idesc,
                             (s >= NMMA || i != 0));
                umma_commit(&sm->mdone[slot]);
                c.mma_slot = slot;
                c.mma_par = par(s);
            }
        }
    } else {
        const int dt = tid - 32 * (NMMA + 1);   // 0 .. 32 * NDQ - 1
        const int kc0 = dt / N, n0 = dt - kc0 * N, dkc = (32 * NDQ) / N, dn = (32 * NDQ) - dkc * N;
        for (int s = 0; s < S; ++s) {
            const int slot = s % nr;
            ok = mbar_wait_b(c, &sm->full[slot], par(s), 210 + slot);
            if (!ok) break;
            uint8_t* bb = sm->ring + slot * SB + AB;
            const uint8_t* raw = bb + BB;
            // item (kc, n): 8 int8 -> one 16-byte row of a core matrix
            // item i = kc * N + n walks by 32 * NDQ: (kc, n) advanced without a division
            for (int kc = kc0, n = n0; kc < KS / 8;) {
                const uint2 w8 = *reinterpret_cast<const uint2*>(raw + (n >> 4) * (TROWS * KS) + kc * 128 + (n & 15) * 8);
                uint4 o;
                i8x4_to_f16x4(w8.x, o.x, o.y);
                i8x4_to_f16x4(w8.y, o.z, o.w);
                *reinterpret_cast<uint4*>(bb + kc * (N * 16) + n * 16) = o;
                n += dn;
                kc += dkc;
                if (n >= N) { n -= N; ++kc; }
            }
            fence_proxy_async();   // generic writes above -> tensor-core (async proxy) reads
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm->deq[slot]);
        }
    }
    // every slot was used u_i times in this GEMM: flip the parities of the odd ones
    uint32_t flip = 0u;
    for (int i = 0; i < nr; ++i)
        if (((S / nr) + (i < S % nr ? 1 : 0)) & 1) flip |= 1u << i;
    c.upar = par0 ^ flip;
    // each issuer's tcgen05 operations complete in order: its last commit covers all of its MMAs
    for (int s = max(0, S - NMMA); s < S && ok; ++s) ok = mbar_wait_b(c, &sm->mdone[s % nr], par(s), 230);
    ok = __syncthreads_and(ok);
    if (!ok) return false;
    c.pend = 0u;
    c.mma_slot = -1;
    tc_fence_after();
    float* Ew = reinterpret_cast<float*>(sm->ring);
    ldE = N + 4;
    const int q = warp & 3;   // tcgen05.ld: warp w reaches TMEM lanes 32 (w % 4) .. + 31; rows 0..63 only
    for (int c8 = q < XC / 512 ? warp >> 2 : N / 8; c8 < N / 8; c8 += NW / 4) {
        float v[8];
        tmem_ld8(c.tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(c8 * 8), v);
#pragma unroll
        for (int k = 1; k < NMMA; ++k) {
            float u[8];
            tmem_ld8(c.tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(k * ACC_COLS + c8 * 8), u);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] += u[i];
        }
        float* dst = Ew + (size_t)(32 * q + lane) * ldE + c8 * 8;
        *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
    tc_fence_before();
    __syncthreads();
    E = Ew;
    return true;
}

// Runs one CTA's row tiles [T0, T1) in passes of at most MAX_TILES_PASS tiles:
// slab width 128 when all tiles fit one pass of at most 5 tiles, else 64.
// epi(E, ldE, g0, nt) consumes each pass's accumulator (tiles g0 .. g0 + nt).
template <class TilePtr, class Epi>
__device__ bool tc_rows(Ctx& c, const uint8_t* xa, int K, int T0, int T1, TilePtr tile_ptr, Epi epi,
                        const int8_t* slab_base = nullptr, int slab_ntm = 0, int slab_k = KBLK) {
    const int n = T1 - T0;
    if (n <= 0) return true;
    const float* E = nullptr;
    int ldE = 0;
    bool ok = true;
    const int passes = (n + MAX_TILES_PASS - 1) / MAX_TILES_PASS;
    for (int p = 0; p < passes && ok; ++p) {
        const int g0 = T0 + split_lo(n, passes, p), g1 = T0 + split_lo(n, passes, p + 1);
#ifndef MQB_KSL
#define MQB_KSL 256
#endif
        if (slab_ntm > 0 && slab_k == 256)
            ok = tc_gemm<256>(c, xa, K, g1 - g0, [&](int j) { return tile_ptr(g0 + j); }, E, ldE, slab_base, slab_ntm, g0);
        else if (slab_ntm > 0)
            ok = tc_gemm<64>(c, xa, K, g1 - g0, [&](int j) { return tile_ptr(g0 + j); }, E, ldE, slab_base, slab_ntm, g0);
        else if (MQB_KSL >= 512 && SlabGeom<512>::A_BYTES + 3 * (g1 - g0) * TROWS * 512 <= RING / 2 && K % 512 == 0)
            ok = tc_gemm<512>(c, xa, K, g1 - g0, [&](int j) { return tile_ptr(g0 + j); }, E, ldE);
        else if (MQB_KSL >= 256 && SlabGeom<256>::A_BYTES + 3 * (g1 - g0) * TROWS * 256 <= RING / 3)
            ok = tc_gemm<256>(c, xa, K, g1 - g0, [&](int j) { return tile_ptr(g0 + j); }, E, ldE);
        else if (g1 - g0 <= 5)
            ok = tc_gemm<128>(c, xa, K, g1 - g0, [&](int j) { return tile_ptr(g0 + j); }, E, ldE);
        else
            ok = tc_gemm<64>(c, xa, K, g1 - g0, [&](int j) { return tile_ptr(g0 + j); }, E, ldE);
        if (ok) epi(E, ldE, g0, g1 - g0);
        fence_proxy_async();
        __syncthreads();
    }
    return ok;
}

// Leaving the kernel: wait (bounded) for copies and MMAs still in flight, then free TMEM.
__device__ void drain_and_free(Ctx& c) {
    Smem* sm = c.sm;
    if (threadIdx.x == 0)   // the producer's copies
        for (int s = 0; s < NR; ++s)
            if (c.pend & (1u << s)) mbar_drain(&sm->full[s], (c.ppar >> s) & 1u, c.budget);
    if (threadIdx.x >= 32 && threadIdx.x <= 32 * NMMA && (threadIdx.x & 31) == 0 && c.mma_slot >= 0)   // the MMA issuers' last commits
        mbar_drain(&sm->mdone[c.mma_slot], c.mma_par, c.budget);
    tc_fence_before();
    __syncthreads();
    if ((threadIdx.x >> 5) == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(c.tmem), "r"(TMEM_COLS) : "memory");
    }
}
__device__ void alloc_tmem(Ctx& c) {
    Smem* sm = c.sm;
    if ((threadIdx.x >> 5) == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm->tmem_base)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    c.tmem = sm->tmem_base;
}
__device__ void init_ctx(Ctx& c, Smem* sm, unsigned* ctl, unsigned long long budget) {
    c.sm = sm;
    c.ctl = ctl;
    c.budget = budget;
    c.tmem = 0;
    c.barriers = 0;
    c.upar = 0;
    c.pend = 0;
    c.ppar = 0;
    c.mma_slot = -1;
    c.mma_par = 0;
    c.half = -1;
    if (threadIdx.x == 0) {
        for (int i = 0; i < NR; ++i) { mbar_init(&sm->full[i], 1); mbar_init(&sm->mdone[i], 1); mbar_init(&sm->deq[i], NDQ); }
        for (int i = 0; i < NAW; ++i)
            for (int j = 0; j < NBUF; ++j) mbar_init(&sm->abar[i][j], 1);
        sm->abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i < BMAX; i += NT) sm->tokbest[i] = 0ull;
    __syncthreads();
    alloc_tmem(c);
}

// ---------------------------------------------------------------------------
// Warp-level bf16 MMA pieces for the attention products
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&a)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]) : "r"(addr) : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&a)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]) : "r"(addr) : "memory");
}
// Two floats as bf16x2 (part 0: the bf16 of x; part 1: the bf16 of the remainder).
__device__ __forceinline__ uint32_t bf2_part(float x, float y, int part) {
    __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    if (part) {
        const float2 f = __bfloat1622float2(h);
        h = __floats2bfloat162_rn(x - f.x, y - f.y);
    }
    return *reinterpret_cast<const uint32_t*>(&h);
}

// ---------------------------------------------------------------------------
// Attention: one warp per (sequence, KV head, split)
// ---------------------------------------------------------------------------
// Work split: the (sequence, KV head, position) triples of a step, flattened
// sequence-major as f = seqoff[b] + kvh * cache_len_b + p, are cut into equal
// ranges of Q (a multiple of 16, >= 256) -- one range per warp of the grid.  A
// range that crosses (b, kvh) boundaries yields one partial per piece; the piece
// starting at f of (b, kvh) has index f / Q - F / Q, F = the flattened start of
// (b, kvh).  Every CTA derives the same cut from the positions, so the merge
// needs no bookkeeping.
__device__ __forceinline__ int nseg_of(int F, int c_len, int Q) { return (F + c_len - 1) / Q - F / Q + 1; }

// QK-RMSNorm + split-half RoPE of one 128-dim head (lane holds dims lane + 32j; partners j, j + 2).
__device__ __forceinline__ void norm_rope(const float* raw, const __nv_bfloat16* nw, const __nv_bfloat16* cosr,
                                          const __nv_bfloat16* sinr, int lane, float out[4]) {
    float v[4], ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) { v[j] = __ldcg(raw + lane + 32 * j); ss += v[j] * v[j]; }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)HD + RMS_EPS);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = v[j] * r * __bfloat162float(nw[lane + 32 * j]);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int i = lane + 32 * j;
        out[j] = v[j] * __bfloat162float(cosr[i]) - v[j + 2] * __bfloat162float(sinr[i]);
        out[j + 2] = v[j] * __bfloat162float(sinr[i + 64]) + v[j + 2] * __bfloat162float(cosr[i + 64]);
    }
}

// Prefill: K (normed, rotated) and V of row b's token for KV head kvh into the
// shared cache at the row's position (one warp).
__device__ void kv_write_item(const Params& P, int l, int b, int kvh) {
    const int lane = threadIdx.x & 31;
    const int pos = P.positions[b];
    const float* qkv = P.qkv + (size_t)b * QKV_ROWS;
    float o[4];
    norm_rope(qkv + QSZ + kvh * HD, (const __nv_bfloat16*)P.layers[l].k_norm_weight, P.cos_t + (size_t)pos * HD,
              P.sin_t + (size_t)pos * HD, lane, o);
    const size_t off = (((size_t)l * NKVH + kvh) * (size_t)P.max_seq + pos) * HD;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int i = lane + 32 * j;
        reinterpret_cast<uint16_t*>(P.kc)[off + i] = (uint16_t)f32_to_bf16_bits(o[j]);
        reinterpret_cast<uint16_t*>(P.vc)[off + i] = (uint16_t)f32_to_bf16_bits(__ldcg(qkv + QSZ + KVSZ + kvh * HD + i));
    }
}

// Positions [pa, pb) of (b, kvh) -> partial s.  The piece with pb = cache_len
// owns the current position: it writes K/V there and takes it from registers.
__device__ void attn_item(Ctx& c, const Params& P, int l, int b, int kvh, int pa, int pb, int s, uint32_t& ause,
                          uint32_t& apend) {
    Smem* sm = c.sm;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = P.positions[b];
    const int c_len = pos + 1;
    const int p0 = pa;
    const bool owner = pb == c_len && !P.prefill; // prefill: this step's K/V are in the cache already
    const int p1 = owner ? pos : pb;              // cached positions [p0, p1)
    const int cb = P.prefill ? 0 : b;             // cache row
    const LayerWeights& w = P.layers[l];
    const float* qkv = P.qkv + (size_t)b * QKV_ROWS;
    const __nv_bfloat16* cosr = P.cos_t + (size_t)pos * HD;
    const __nv_bfloat16* sinr = P.sin_t + (size_t)pos * HD;
    float* q = sm->a.q[warp][0];
#pragma unroll
    for (int hq = 0; hq < 2; ++hq) {
        float o[4];
        norm_rope(qkv + (2 * kvh + hq) * HD, (const __nv_bfloat16*)w.q_norm_weight, cosr, sinr, lane, o);
#pragma unroll
        for (int j = 0; j < 4; ++j) q[hq * HD + lane + 32 * j] = o[j];
    }
    uint16_t kcur[4], vcur[4];
    if (owner) {
        float o[4];
        norm_rope(qkv + QSZ + kvh * HD, (const __nv_bfloat16*)w.k_norm_weight, cosr, sinr, lane, o);
        const size_t off = ((((size_t)cb * P.L + l) * NKVH + kvh) * (size_t)P.max_seq + pos) * HD;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = lane + 32 * j;
            kcur[j] = (uint16_t)f32_to_bf16_bits(o[j]);
            vcur[j] = (uint16_t)f32_to_bf16_bits(__ldcg(qkv + QSZ + KVSZ + kvh * HD + i));
            reinterpret_cast<uint16_t*>(P.kc)[off + i] = kcur[j];
            reinterpret_cast<uint16_t*>(P.vc)[off + i] = vcur[j];
        }
    }
    __syncwarp();
    // Tensor-core flash-decode (mma.sync m16n8k16 bf16, fp32 accumulation) over
    // 16-position chunks, both GQA heads at once:
    //   S[16 pos x 8] = K[16 x 128] * Qt, Q columns = q0 hi, q1 hi, q0 lo, q1 lo
    //   (bf16 hi + lo parts of the fp32 q, so the scores carry ~16 bits of q);
    //   Ot[128 dims x 8] += Vt * Pt, P columns the same hi/lo split of exp(s - m).
    // K tiles come through ldmatrix, V tiles through ldmatrix.trans.
    static_assert(ACH == 16, "tensor-core attention: 16-position chunks");
    const int g = lane >> 2, t = lane & 3;
    const float scale = P.attn_scale;
    uint32_t qb[HD / 16][2];
#pragma unroll
    for (int k8 = 0; k8 < HD / 16; ++k8)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const int d = 16 * k8 + 8 * hf + 2 * t;
            qb[k8][hf] = g < 4 ? bf2_part(q[(g & 1) * HD + d], q[(g & 1) * HD + d + 1], g >> 1) : 0u;
        }
    float acc[HD / 16][4];
#pragma unroll
    for (int mt = 0; mt < HD / 16; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
    float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;   // running max / sum of heads 0 and 1
    // A chunk buffer holds K then V, each as two 16-row x 128-byte boxes (dims 0..63, 64..127) in the TMA
    // 128-byte swizzle: 16-byte unit u of row r sits at unit u ^ (r & 7).
    auto chunk = [&](uint8_t* buf, int n) {
        const uint32_t kbase = smem_u32(buf), vbase = kbase + ACH * HD * 2;
        if (n < ACH) {   // V rows past n must be finite (P is 0 there, and 0 * NaN would poison the sums)
            uint4* zv = reinterpret_cast<uint4*>(buf + ACH * HD * 2);
            for (int i = lane; i < 2 * (ACH - n) * 8; i += 32) {
                const int bx = i / ((ACH - n) * 8), r = n + (i / 8) % (ACH - n);
                zv[bx * ACH * 8 + r * 8 + (i & 7)] = make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
        }
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        const int sw = lane & 7;   // = row & 7 for the rows this lane addresses
        const uint32_t ka = kbase + ((lane & 7) + ((lane >> 3) & 1) * 8) * 128;
#pragma unroll
        for (int k8 = 0; k8 < HD / 16; ++k8) {
            uint32_t a[4];
            ldsm_x4(a, ka + (k8 >> 2) * (ACH * 128) + ((((2 * k8 + (lane >> 4)) & 7) ^ sw) << 4));
            mma16816(c, a, qb[k8][0], qb[k8][1]);
        }
        // hi + lo columns: lanes t = 0 hold (q0 hi, q1 hi), t = 1 (q0 lo, q1 lo)
        float s0 = c[0] + __shfl_xor_sync(0xffffffffu, c[0], 1);   // position g, head 0
        float s1 = c[1] + __shfl_xor_sync(0xffffffffu, c[1], 1);   // position g, head 1
        float s2 = c[2] + __shfl_xor_sync(0xffffffffu, c[2], 1);   // position g + 8, head 0
        float s3 = c[3] + __shfl_xor_sync(0xffffffffu, c[3], 1);   // position g + 8, head 1
        const bool v0 = g < n, v1 = g + 8 < n;
        s0 = v0 ? s0 * scale : -INFINITY; s1 = v0 ? s1 * scale : -INFINITY;
        s2 = v1 ? s2 * scale : -INFINITY; s3 = v1 ? s3 * scale : -INFINITY;
        float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
        }
        mx0 = __shfl_sync(0xffffffffu, mx0, 0);   // lanes t = 0 reduced the real scores
        mx1 = __shfl_sync(0xffffffffu, mx1, 0);
        const float n0 = fmaxf(mA, mx0), n1 = fmaxf(mB, mx1);
        const float cf0 = expf(mA - n0), cf1 = expf(mB - n1);   // 0 while m is still -inf
        const float e0 = v0 ? expf(s0 - n0) : 0.f, e1 = v0 ? expf(s1 - n1) : 0.f;
        const float e2 = v1 ? expf(s2 - n0) : 0.f, e3 = v1 ? expf(s3 - n1) : 0.f;
        float es0 = e0 + e2, es1 = e1 + e3;
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            es0 += __shfl_xor_sync(0xffffffffu, es0, o);
            es1 += __shfl_xor_sync(0xffffffffu, es1, o);
        }
        lA = lA * cf0 + __shfl_sync(0xffffffffu, es0, 0);
        lB = lB * cf1 + __shfl_sync(0xffffffffu, es1, 0);
        mA = n0;
        mB = n1;
#pragma unroll
        for (int mt = 0; mt < HD / 16; ++mt) { acc[mt][0] *= cf0; acc[mt][1] *= cf1; acc[mt][2] *= cf0; acc[mt][3] *= cf1; }
        // Pt fragment of column g (< 4: head g & 1, hi/lo part g >> 1): positions 2t, 2t + 1, 2t + 8, 2t + 9,
        // held by lanes 4 * (2t) and 4 * (2t + 1)
        const float a0_ = __shfl_sync(0xffffffffu, e0, 8 * t), a1_ = __shfl_sync(0xffffffffu, e1, 8 * t);
        const float a2_ = __shfl_sync(0xffffffffu, e2, 8 * t), a3_ = __shfl_sync(0xffffffffu, e3, 8 * t);
        const float b0_ = __shfl_sync(0xffffffffu, e0, 8 * t + 4), b1_ = __shfl_sync(0xffffffffu, e1, 8 * t + 4);
        const float b2_ = __shfl_sync(0xffffffffu, e2, 8 * t + 4), b3_ = __shfl_sync(0xffffffffu, e3, 8 * t + 4);
        const bool h1 = g & 1;
        uint32_t pb0 = 0u, pb1 = 0u;
        if (g < 4) {
            pb0 = bf2_part(h1 ? a1_ : a0_, h1 ? b1_ : b0_, g >> 1);
            pb1 = bf2_part(h1 ? a3_ : a2_, h1 ? b3_ : b2_, g >> 1);
        }
        const uint32_t va = vbase + ((lane & 7) + (lane >> 4) * 8) * 128;
#pragma unroll
        for (int mt = 0; mt < HD / 16; ++mt) {
            uint32_t a[4];
            ldsm_x4_t(a, va + (mt >> 2) * (ACH * 128) + ((((2 * mt + ((lane >> 3) & 1)) & 7) ^ sw) << 4));
            mma16816(acc[mt], a, pb0, pb1);
        }
    };
    // cached positions [p0, p1) in ACH-position chunks, NBUF in flight per warp
    const int head = ((cb * P.L + l) * NKVH + kvh) * P.max_seq;   // first tensor row of this (sequence, layer, head)
    const int nch = (p1 - p0 + ACH - 1) / ACH;
    auto issue = [&](int ci) {   // lane 0
        const int row = head + p0 + ACH * ci;   // a whole box is copied; rows past the range are masked
        const int bi = ci % NBUF;
        uint8_t* buf = sm->a.kv[warp][bi];
        uint64_t* bar = &sm->abar[warp][bi];
        fence_proxy_async();
        mbar_arrive_expect_tx(bar, 2u * ACH * HD * 2);
        tma_load_2d(buf, &P.tm_k, 0, row, bar);
        tma_load_2d(buf + ACH * 128, &P.tm_k, 64, row, bar);
        tma_load_2d(buf + ACH * HD * 2, &P.tm_v, 0, row, bar);
        tma_load_2d(buf + ACH * HD * 2 + ACH * 128, &P.tm_v, 64, row, bar);
    };
    __syncwarp();
    for (int ci = 0; ci < min(NBUF, nch); ++ci) {
        if (lane == 0) issue(ci);
        apend |= 1u << ci;
    }
    for (int ci = 0; ci < nch; ++ci) {
        const int bs = ci % NBUF;
        if (!mbar_wait_b(c, &sm->abar[warp][bs], (ause >> bs) & 1u, 300)) return;
        apend &= ~(1u << bs);
        ause ^= 1u << bs;
        chunk(sm->a.kv[warp][bs], min(ACH, p1 - p0 - ACH * ci));
        __syncwarp();
        if (ci + NBUF < nch) {
            if (lane == 0) issue(ci + NBUF);
            apend |= 1u << bs;
        }
    }
    if (owner) {  // the current position from registers (all buffers are free now)
        // row 0 of a box is unswizzled: dim i sits at box i / 64, byte 2 (i % 64)
        uint16_t* kw = reinterpret_cast<uint16_t*>(sm->a.kv[warp][0]);
        uint16_t* vw = reinterpret_cast<uint16_t*>(sm->a.kv[warp][0] + ACH * HD * 2);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = lane + 32 * j, o = (i >> 6) * (ACH * 64) + (i & 63);
            kw[o] = kcur[j];
            vw[o] = vcur[j];
        }
        __syncwarp();
        chunk(sm->a.kv[warp][0], 1);
    }
    float* out = P.part + (((size_t)b * NKVH + kvh) * MAX_SPLITS_B + s) * PARTW;
#pragma unroll
    for (int mt = 0; mt < HD / 16; ++mt) {
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = acc[mt][j] + __shfl_xor_sync(0xffffffffu, acc[mt][j], 1);   // hi + lo
        if (t == 0) {
            out[16 * mt + g] = o[0];
            out[HD + 16 * mt + g] = o[1];
            out[16 * mt + g + 8] = o[2];
            out[HD + 16 * mt + g + 8] = o[3];
        }
    }
    if (lane == 0) { out[2 * HD] = mA; out[2 * HD + 1] = mB; out[2 * HD + 2] = lA; out[2 * HD + 3] = lB; }
}


// One warp per (sequence, q head): merges the splits into the O-projection
// operand (this lane's 4 columns = half of one 8-wide k column row).
__device__ void merge_item(const Smem* sm, const Params& P, int b, int qh) {
    const int lane = threadIdx.x & 31;
    const int kvh = qh >> 1, hh = qh & 1;
    const int c_len = P.positions[b] + 1;
    const int ns = nseg_of(sm->seqoff[b] + kvh * c_len, c_len, sm->segq);
    const float* base = P.part + ((size_t)b * NKVH + kvh) * MAX_SPLITS_B * PARTW;
    // one online pass over the partials (loads do not depend on the running state)
    float M = -INFINITY, L = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int s = 0; s < ns; ++s) {
        const float* ps = base + (size_t)s * PARTW;
        const float ms = __ldcg(ps + 2 * HD + hh), ls = __ldcg(ps + 2 * HD + 2 + hh);
        const float4 a = __ldcg(reinterpret_cast<const float4*>(ps + hh * HD + 4 * lane));
        const float Mn = fmaxf(M, ms);
        const float cprev = expf(M - Mn), cs = expf(ms - Mn);
        L = L * cprev + ls * cs;
        o[0] = o[0] * cprev + a.x * cs; o[1] = o[1] * cprev + a.y * cs;
        o[2] = o[2] * cprev + a.z * cs; o[3] = o[3] * cprev + a.w * cs;
        M = Mn;
    }
    const float inv = XS_ACT / L;
    uint32_t w[2];
    bool ok = true;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float x0 = o[2 * i] * inv, x1 = o[2 * i + 1] * inv;
        ok &= fabsf(x0) <= 65504.f && fabsf(x1) <= 65504.f;
        const __half2 h = __floats2half2_rn(x0, x1);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    const int k0 = qh * HD + 4 * lane;
    *reinterpret_cast<uint2*>(P.xa_o + (size_t)(b / HROWS) * (QSZ / 8) * HXCOL + (size_t)(k0 >> 3) * HXCOL +
                              (b % HROWS) * 16 + (k0 & 7) * 2) = make_uint2(w[0], w[1]);
    if (!ok) range_fail(P.ctl, 3);
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// ---------------------------------------------------------------------------
// The step kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT, 1) batch_kernel(const __grid_constant__ Params P) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the 128-byte-swizzled TMA boxes need 1024-byte aligned destinations: one spare KB is allocated
    Smem* sm = reinterpret_cast<Smem*>(smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
    Ctx c;
    init_ctx(c, sm, P.ctl, P.budget_ns);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = gridDim.x, cta = blockIdx.x;
    const int B = P.B;
    // Every CTA validates the per-sequence inputs before touching memory with them.
    for (int t = threadIdx.x; t < B; t += NT) {
        const int tok = P.tokens_in[t], pos = P.positions[t];
        if (tok < 0 || tok >= VOCAB) fail(c, MQ_DEV_BAD_TOKEN, t);
        if (pos < 0 || pos >= P.max_seq) fail(c, MQ_DEV_BAD_POSITION, t);
    }
    if (threadIdx.x == 0) {
        int o = 0;
        for (int t = 0; t < B; ++t) { sm->seqoff[t] = o; o += NKVH * (P.positions[t] + 1); }
        sm->seqoff[B] = o;
        const int W = nb * NAW;
        int q = (o + W - 1) / W;
        q = (q + 15) & ~15;
        sm->segq = q < 256 ? 256 : q;
    }
    __syncthreads();
    uint32_t ause = 0u;      // bit i: parity of the next use of this warp's KV buffer i
    uint32_t apend = 0u;     // buffers with a KV-chunk copy not waited for
    bool ok = !*(volatile int*)&sm->abort_flag;
    // ---- embedding rows -> h and the layer-0 QKV operand ----
    if (ok) {
        const int T0 = split_lo(HT, nb, cta), T1 = split_lo(HT, nb, cta + 1);
        const __nv_bfloat16* nw = (const __nv_bfloat16*)P.layers[0].input_layernorm_weight;
        for (int i = threadIdx.x; i < B * (T1 - T0); i += NT) {
            const int t = i % B, g = T0 + i / B, row = TROWS * g;
            float v[16], wv[16], x[16], ss = 0.f;
            load16_bf16(P.embed + (size_t)P.tokens_in[t] * HIDDEN, row, v);
            load16_bf16(nw, row, wv);
#pragma unroll
            for (int k = 0; k < 16; ++k) { ss += v[k] * v[k]; x[k] = v[k] * wv[k]; }
            store16(P.h + (size_t)t * HIDDEN, row, v);
            P.ss_a[g * BMAX + t] = ss;
            if (!(put_x8(P.xa_qkv, t, row, x, XS_NORM) & put_x8(P.xa_qkv, t, row + 8, x + 8, XS_NORM)))
                range_fail(P.ctl, 0);
        }
    }
    stamp(P, 0);
    ok = grid_barrier(c, 0) && ok;
    for (int l = 0; l < P.L && ok; ++l) {
        const LayerWeights& w = P.layers[l];
        const ScalePointers& sc = P.scales[l];
        // ---- QKV ----
        {
            compute_rstd(sm, P.ss_a, B);
            const int NTQ = QKV_ROWS / TROWS;
            const int T0 = split_lo(NTQ, nb, cta), T1 = split_lo(NTQ, nb, cta + 1);
            const int8_t* wq = (const int8_t*)w.q_proj_weight;
            const int8_t* wk = (const int8_t*)w.k_proj_weight;
            const int8_t* wv = (const int8_t*)w.v_proj_weight;
            const float* sq = sc.q_scale; const float* sk = sc.k_scale; const float* sv = sc.v_scale;
            auto tp = [&](int g) -> const int8_t* {
                return g < QSZ / TROWS ? wq + (size_t)g * TROWS * HIDDEN
                       : g < (QSZ + KVSZ) / TROWS ? wk + (size_t)(g - QSZ / TROWS) * TROWS * HIDDEN
                                                  : wv + (size_t)(g - (QSZ + KVSZ) / TROWS) * TROWS * HIDDEN;
            };
            ok = tc_rows(c, P.xa_qkv, HIDDEN, T0, T1, tp, [&](const float* E, int ldE, int g0, int nt) {
                     for (int i = threadIdx.x; i < B * nt; i += NT) {
                         const int t = i % B, g = g0 + i / B, row = TROWS * g;
                         float v[16];
                         erow16(E, ldE, t, TROWS * (g - g0), 1.0f / XS_NORM, v);
                         const float* s_ = row < QSZ ? sq + row : row < QSZ + KVSZ ? sk + (row - QSZ) : sv + (row - QSZ - KVSZ);
                         const float r = sm->rstd[t];
#pragma unroll
                         for (int k = 0; k < 16; ++k) v[k] = v[k] * __ldg(s_ + k) * r;
                         store16(P.qkv + (size_t)t * QKV_ROWS, row, v);
                     }
                 }, wq, NTQ, 256) && ok;
        }
        stamp(P, l * 8 + 1);
        if (!grid_barrier(c, 1)) { ok = false; break; }
        if (P.prefill) {   // every row's K/V in the cache before any attention reads it
            for (int it = cta * NW + warp; it < B * NKVH; it += nb * NW) kv_write_item(P, l, it / NKVH, it % NKVH);
            if (!grid_barrier(c, 8)) { ok = false; break; }
        }
        // ---- attention ----
        {
            const int Q = sm->segq, T = sm->seqoff[B];
            int f = warp < NAW ? (cta * NAW + warp) * Q : T;
            const int fe = min(T, f + Q);
            int b = 0;
            while (f < fe) {
                while (sm->seqoff[b + 1] <= f) ++b;
                const int c_len = P.positions[b] + 1;
                const int r = f - sm->seqoff[b];
                const int kvh = r / c_len, pa = r - kvh * c_len;
                const int pb = min(c_len, pa + (fe - f));
                const int F = sm->seqoff[b] + kvh * c_len;
                attn_item(c, P, l, b, kvh, pa, pb, f / Q - F / Q, ause, apend);
                if (apend) break;
                f += pb - pa;
            }
        }
        stamp(P, l * 8 + 2);
        if (!grid_barrier(c, 2)) { ok = false; break; }
        // ---- merge ----
        for (int it = cta * NW + warp; it < B * NQH; it += nb * NW) merge_item(sm, P, it / NQH, it % NQH);
        stamp(P, l * 8 + 3);
        if (!grid_barrier(c, 3)) { ok = false; break; }
        // ---- O + residual -> act, GU operand ----
        // Units (16-row tile g, token half h): each CTA reads the half of the operand
        // it needs, and 128 CTAs share the work instead of 64.
        {
            const int U0 = split_lo(2 * HT, nb, cta), U1 = split_lo(2 * HT, nb, cta + 1);
            const int8_t* wo = (const int8_t*)w.o_proj_weight;
            const __nv_bfloat16* pw = (const __nv_bfloat16*)w.post_attn_layernorm_weight;
            const float* so = sc.o_scale;
            for (int u = U0; u < U1 && ok; ++u) {
                const int g = u >> 1, h = u & 1, nt_h = min(HROWS, B - h * HROWS);
                if (nt_h <= 0) continue;
                c.half = h;
                ok = tc_rows(c, P.xa_o, QSZ, g, g + 1, [&](int gg) { return wo + (size_t)gg * TROWS * QSZ; },
                             [&](const float* E, int ldE, int, int) {
                                 for (int r = threadIdx.x; r < nt_h; r += NT) {
                                     const int t = h * HROWS + r, row = TROWS * g;
                                     float v[16], hv[16], wv[16], x[16], ss = 0.f;
                                     erow16(E, ldE, r, 0, 1.0f / XS_ACT, v);
                                     load16(P.h + (size_t)t * HIDDEN, row, hv);
                                     load16_bf16(pw, row, wv);
#pragma unroll
                                     for (int k = 0; k < 16; ++k) {
                                         v[k] = v[k] * __ldg(so + row + k) + hv[k];
                                         ss += v[k] * v[k];
                                         x[k] = v[k] * wv[k];
                                     }
                                     store16(P.act + (size_t)t * HIDDEN, row, v);
                                     P.ss_b[g * BMAX + t] = ss;
                                     if (!(put_x8(P.xa_gu, t, row, x, XS_NORM) & put_x8(P.xa_gu, t, row + 8, x + 8, XS_NORM)))
                                         range_fail(P.ctl, 4);
                                 }
                             }, wo, HT, 256) && ok;
                c.half = -1;
            }
        }
        stamp(P, l * 8 + 4);
        if (!grid_barrier(c, 4)) { ok = false; break; }
        // ---- gate/up + SiLU -> DOWN operand ----
        {
            compute_rstd(sm, P.ss_b, B);
            const int NP = INTER / TROWS;
            const int P0 = split_lo(NP, nb, cta), np = split_lo(NP, nb, cta + 1) - P0;
            const int8_t* wg = (const int8_t*)w.gate_proj_weight;
            const float* sg = sc.gate_scale; const float* su = sc.up_scale;
            // fused gate/up matrix, pair-interleaved: tile 2p = gate rows of pair p, 2p + 1 = up rows
            // (one pass: np <= 2); this CTA's pairs are the contiguous tiles [2 P0, 2 P0 + 2 np)
            ok = tc_rows(c, P.xa_gu, HIDDEN, 2 * P0, 2 * (P0 + np),
                         [&](int g) { return wg + (size_t)g * TROWS * HIDDEN; },
                         [&](const float* E, int ldE, int, int) {
                             for (int i = threadIdx.x; i < B * np; i += NT) {
                                 const int t = i % B, jp = i / B, row = TROWS * (P0 + jp);
                                 float gv[16], uv[16], m[16];
                                 erow16(E, ldE, t, TROWS * (2 * jp), 1.0f / XS_NORM, gv);
                                 erow16(E, ldE, t, TROWS * (2 * jp + 1), 1.0f / XS_NORM, uv);
                                 const float r = sm->rstd[t];
#pragma unroll
                                 for (int k = 0; k < 16; ++k) {
                                     const float gd = gv[k] * __ldg(sg + row + k) * r;
                                     const float ud = uv[k] * __ldg(su + row + k) * r;
                                     m[k] = gd / (1.0f + expf(-gd)) * ud;
                                 }
                                 if (!(put_x8h(P.xa_dn, INTER, t, row, m, XS_ACT) & put_x8h(P.xa_dn, INTER, t, row + 8, m + 8, XS_ACT)))
                                     range_fail(P.ctl, 5);
                             }
                         }, wg, 2 * NP, 256) && ok;
        }
        stamp(P, l * 8 + 5);
        if (!grid_barrier(c, 5)) { ok = false; break; }
        // ---- down + residual -> h, next QKV (or LM-head) operand (units as for O) ----
        {
            const int U0 = split_lo(2 * HT, nb, cta), U1 = split_lo(2 * HT, nb, cta + 1);
            const int8_t* wd = (const int8_t*)w.down_proj_weight;
            const float* sd = sc.down_scale;
            const __nv_bfloat16* nn =
                l + 1 < P.L ? (const __nv_bfloat16*)P.layers[l + 1].input_layernorm_weight : P.final_norm;
            for (int u = U0; u < U1 && ok; ++u) {
                const int g = u >> 1, h = u & 1, nt_h = min(HROWS, B - h * HROWS);
                if (nt_h <= 0) continue;
                c.half = h;
                ok = tc_rows(c, P.xa_dn, INTER, g, g + 1, [&](int gg) { return wd + (size_t)gg * TROWS * INTER; },
                             [&](const float* E, int ldE, int, int) {
                                 for (int r = threadIdx.x; r < nt_h; r += NT) {
                                     const int t = h * HROWS + r, row = TROWS * g;
                                     float v[16], av[16], wv[16], x[16], ss = 0.f;
                                     erow16(E, ldE, r, 0, 1.0f / XS_ACT, v);
                                     load16(P.act + (size_t)t * HIDDEN, row, av);
                                     load16_bf16(nn, row, wv);
#pragma unroll
                                     for (int k = 0; k < 16; ++k) {
                                         v[k] = bf16r(v[k] * __ldg(sd + row + k) + av[k]);
                                         ss += v[k] * v[k];
                                         x[k] = v[k] * wv[k];
                                     }
                                     store16(P.h + (size_t)t * HIDDEN, row, v);
                                     P.ss_a[g * BMAX + t] = ss;
                                     if (!(put_x8(P.xa_qkv, t, row, x, XS_NORM) & put_x8(P.xa_qkv, t, row + 8, x + 8, XS_NORM)))
                                         range_fail(P.ctl, 6);
                                 }
                             }, wd, HT, 256) && ok;
                c.half = -1;
            }
        }
        stamp(P, l * 8 + 6);
        if (!grid_barrier(c, 6)) { ok = false; break; }
    }
    // ---- LM head + per-sequence argmax ----
    if (ok) {
        compute_rstd(sm, P.ss_a, B);
        const int NTL = VOCAB / TROWS;
        const int T0 = P.lm_tile0 + split_lo(P.lm_tiles, nb, cta), T1 = P.lm_tile0 + split_lo(P.lm_tiles, nb, cta + 1);
        ok = tc_rows(c, P.xa_qkv, HIDDEN, T0, T1, [&](int g) { return P.lm_w + (size_t)g * TROWS * HIDDEN; },
                     [&](const float* E, int ldE, int g0, int nt) {
                         for (int i = threadIdx.x; i < B * nt; i += NT) {
                             const int t = i % B, g = g0 + i / B, row = TROWS * g;
                             float v[16];
                             erow16(E, ldE, t, TROWS * (g - g0), 1.0f / XS_NORM, v);
                             const float r = sm->rstd[t];
                             unsigned long long best = 0ull;
#pragma unroll
                             for (int k = 0; k < 16; ++k) {
                                 v[k] = v[k] * __ldg(P.lm_scale + row + k) * r;
                                 const unsigned long long key = (((unsigned long long)float_order_key(v[k])) << 32) |
                                                                (uint32_t)(~(uint32_t)(row + k));
                                 best = key > best ? key : best;
                             }
                             if (P.logits) store16(P.logits + (size_t)t * VOCAB, row, v);
                             atomicMax(&sm->tokbest[t], best);
                         }
                     }, P.lm_w, NTL) && ok;
        __syncthreads();
        for (int t = threadIdx.x; t < B; t += NT) atomicMax(&P.best[t], sm->tokbest[t]);
    }
    stamp(P, P.L * 8 + 6);
    grid_barrier(c, 7);
    stamp(P, P.L * 8 + 7);
    if (cta == 0) {
        const bool err = ld_relaxed32(&P.ctl[2]) != 0;
        for (int t = threadIdx.x; t < B; t += NT) {
            const unsigned long long k = __ldcg(P.best + t);
            if (P.keys_out)   // (logit order << 32 | ~row) with the sign bit flipped: a signed max-reduction keeps the order
                P.keys_out[t] = err ? (long long)0x8000000000000000ull : (long long)(k ^ 0x8000000000000000ull);
            else
                P.tokens_out[t] = (err || k == 0ull) ? -1 : (int)(~(uint32_t)k);
            P.best[t] = 0ull;
            if (!err) P.positions[t] += 1;
        }
    }
    if (lane == 0 && warp < NAW)
        for (int i = 0; i < NBUF; ++i)
            if (apend & (1u << i)) mbar_drain(&sm->abar[warp][i], (ause >> i) & 1u, P.budget_ns);
    drain_and_free(c);
    __syncthreads();
    if (threadIdx.x == 0) {  // the last CTA out resets the barrier counter for the next launch
        __threadfence();
        const unsigned old = atomicAdd(&P.ctl[1], 1u);
        if (old == (unsigned)nb - 1) {
            atomicExch(&P.ctl[0], 0u);
            atomicExch(&P.ctl[1], 0u);
            __threadfence();
        }
    }
}

// ---------------------------------------------------------------------------
// Standalone GEMM through the same tensor-core path (tests, benchmarks):
// y[t][m] = scale[m] * sum_k W[m][k] * x[t][k] for t < B.
// ---------------------------------------------------------------------------
struct MMParams {
    const int8_t* w;       // tile-packed [M/16][K/64] blocks
    const float* scale;
    const uint8_t* xa;     // activation operand (written by xpack_kernel)
    float* y;              // [B][M]
    unsigned int* ctl;
    unsigned long long budget_ns;
    int M, K, B;
};

// x fp32 [B][K] -> activation operand (fp16 rows t < B; rows >= B zero).
__global__ void xpack_kernel(const float* x, uint8_t* xa, int K, int B, unsigned* ctl) {
    const int n = BMAX * (K / 8);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int t = i % BMAX, k0 = 8 * (i / BMAX);
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = t < B ? x[(size_t)t * K + k0 + j] : 0.f;
        if (!put_x8(xa, t, k0, v, 1.0f)) range_fail(ctl, 0);
    }
}

__global__ void __launch_bounds__(NT, 1) matmul_kernel(const MMParams Q) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    Smem* sm = reinterpret_cast<Smem*>(smem_raw);
    Ctx c;
    init_ctx(c, sm, Q.ctl, Q.budget_ns);
    const int NTM = Q.M / TROWS;
    const int T0 = split_lo(NTM, gridDim.x, blockIdx.x), T1 = split_lo(NTM, gridDim.x, blockIdx.x + 1);
    tc_rows(c, Q.xa, Q.K, T0, T1, [&](int g) { return Q.w + (size_t)g * TROWS * Q.K; },
            [&](const float* E, int ldE, int g0, int nt) {
                for (int i = threadIdx.x; i < Q.B * nt; i += NT) {
                    const int t = i % Q.B, g = g0 + i / Q.B, row = TROWS * g;
                    float v[16];
                    erow16(E, ldE, t, TROWS * (g - g0), 1.0f, v);
#pragma unroll
                    for (int k = 0; k < 16; ++k) v[k] *= __ldg(Q.scale + row + k);
                    store16(Q.y + (size_t)t * Q.M, row, v);
                }
            });
    drain_and_free(c);
}

// INT8 [rows][K] -> slab-major packed blocks of bk columns: block (kb, tile) at
// ((kb * rows/16) + tile) * 16 * bk, inside [8-k column][16 rows][8 bytes].
__global__ void pack_slabs_kernel(const int8_t* src, int64_t rows, int K, int64_t src_stride, int bk, int8_t* dst) {
    const int64_t n = rows * (K / 8);
    const int64_t ntiles = rows / TROWS;
    const int U = 2 * bk;   // 8-byte units per block
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t blk = i / U;
        const int u = (int)(i - blk * U), kc = u >> 4, r = u & 15;
        const int kb = (int)(blk / ntiles);
        const int64_t tile = blk - (int64_t)kb * ntiles;
        const int8_t* s = src + (tile * TROWS + r) * src_stride + (int64_t)kb * bk + kc * 8;
        uint2 v;
        memcpy(&v, s, 8);
        *reinterpret_cast<uint2*>(dst + i * 8) = v;
    }
}

// INT8 [rows][K] (row stride src_stride bytes) -> tile-packed blocks:
// block (tile, kb) at ((tile * K/64) + kb) * 1024, inside [8-k column][16 rows][8 bytes].
__global__ void pack_tiles_kernel(const int8_t* src, int64_t rows, int K, int64_t src_stride, int8_t* dst) {
    const int64_t n = rows * (K / 8);   // 8-byte units
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t blk = i >> 7;              // 128 units per block
        const int u = (int)(i & 127), kc = u >> 4, r = u & 15;
        const int nkb = K / KBLK;
        const int64_t tile = blk / nkb;
        const int kb = (int)(blk - tile * nkb);
        const int8_t* s = src + (tile * TROWS + r) * src_stride + kb * KBLK + kc * 8;
        uint2 v;
        memcpy(&v, s, 8);
        *reinterpret_cast<uint2*>(dst + i * 8) = v;
    }
}


// ===========================================================================
// Host side
// ===========================================================================
namespace {
struct Layout {
    size_t ctl, best, h, act, qkv, xa_qkv, xa_o, xa_gu, xa_dn, ss_a, ss_b, part, total;
};
size_t up256(size_t x) { return (x + 255) & ~(size_t)255; }
Layout layout(int B) {
    Layout L{};
    size_t o = 0;
    L.ctl = o;    o += up256(4 * sizeof(unsigned));
    L.best = o;   o += up256((size_t)B * sizeof(unsigned long long));
    L.h = o;      o += up256((size_t)B * HIDDEN * 4);
    L.act = o;    o += up256((size_t)B * HIDDEN * 4);
    L.qkv = o;    o += up256((size_t)B * QKV_ROWS * 4);
    L.xa_qkv = o; o += up256((size_t)XCOL * (HIDDEN / 8));
    L.xa_o = o;   o += up256((size_t)XCOL * (QSZ / 8));
    L.xa_gu = o;  o += up256((size_t)XCOL * (HIDDEN / 8));
    L.xa_dn = o;  o += up256((size_t)XCOL * (INTER / 8));
    L.ss_a = o;   o += up256((size_t)HT * BMAX * 4);
    L.ss_b = o;   o += up256((size_t)HT * BMAX * 4);
    L.part = o;   o += up256((size_t)B * NKVH * MAX_SPLITS_B * PARTW * 4);
    L.total = o;
    return L;
}
constexpr int MAX_DEV = 64;
constexpr int MIN_SMS = 96;   // GU: at most 2 gate/up tile pairs per CTA
bool g_attr[MAX_DEV];
int g_sms[MAX_DEV];
bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

cudaError_t setup_device(int& dev) {
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= MAX_DEV) return cudaErrorInvalidDevice;
    if (!g_attr[dev]) {
        if ((e = cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
        if ((e = cudaFuncSetAttribute(batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem) + 1024)) !=
            cudaSuccess)
            return e;
        if ((e = cudaFuncSetAttribute(matmul_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem))) !=
            cudaSuccess)
            return e;
        g_attr[dev] = true;
    }
    return cudaSuccess;
}

// Tensor map of one KV cache as [rows][128] bf16 with 16 x 64 boxes in the 128-byte swizzle.  The
// driver's encoder is fetched through the runtime, so the library does not link libcuda.
cudaError_t encode_cache_map(CUtensorMap* map, const void* base, int rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
        if (e != cudaSuccess) return e;
        if (q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
        encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)HD, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)HD * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)ACH};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}
}  // namespace
}  // namespace batch
}  // namespace mq

using namespace mq;

extern "C" int mq_batch_workspace_bytes(int batch, size_t* bytes) {
    if (batch < 1 || batch > batch::BMAX || !bytes) return MQ_ERR_ARG;
    *bytes = batch::layout(batch).total;
    return 0;
}

extern "C" int mq_pack_weight_tiles(const int8_t* src, int64_t rows, int K, int64_t src_row_stride, int8_t* dst,
                                    cudaStream_t stream) {
    using namespace batch;
    if (!src || !dst || rows <= 0 || K <= 0) return MQ_ERR_ARG;
    if (rows % TROWS != 0 || K % KBLK != 0 || src_row_stride < K || src_row_stride % 8 != 0) return MQ_ERR_SIZE;
    if (((uintptr_t)src & 7u) != 0 || !al16(dst)) return MQ_ERR_ARG;
    const int64_t units = rows * (K / 8);
    const int grid = (int)((units + 255) / 256 < 65536 ? (units + 255) / 256 : 65536);
    pack_tiles_kernel<<<grid, 256, 0, stream>>>(src, rows, K, src_row_stride, dst);
    return (int)cudaGetLastError();
}

extern "C" int mq_pack_weight_slabs(const int8_t* src, int64_t rows, int K, int64_t src_row_stride, int block_k,
                                    int8_t* dst, cudaStream_t stream) {
    using namespace batch;
    if (!src || !dst || rows <= 0 || K <= 0 || (block_k != 64 && block_k != 256)) return MQ_ERR_ARG;
    if (rows % TROWS != 0 || K % block_k != 0 || src_row_stride < K || src_row_stride % 8 != 0) return MQ_ERR_SIZE;
    if (((uintptr_t)src & 7u) != 0 || !al16(dst)) return MQ_ERR_ARG;
    const int64_t units = rows * (K / 8);
    const int grid = (int)((units + 255) / 256 < 65536 ? (units + 255) / 256 : 65536);
    pack_slabs_kernel<<<grid, 256, 0, stream>>>(src, rows, K, src_row_stride, block_k, dst);
    return (int)cudaGetLastError();
}

extern "C" int mq_batch_matmul_workspace_bytes(int K, size_t* bytes) {
    if (!bytes || (K != 1024 && K != 2048 && K != 3072)) return MQ_ERR_ARG;
    *bytes = 256 + (size_t)batch::XCOL * (K / 8);
    return 0;
}

extern "C" int mq_batch_matmul(const int8_t* w_tiles, const float* scale, const float* x, float* y, int M, int K,
                               int B, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    using namespace batch;
    if (!w_tiles || !scale || !x || !y || !workspace) return MQ_ERR_ARG;
    if ((K != 1024 && K != 2048 && K != 3072) || M <= 0 || M % TROWS != 0 || B < 1 || B > BMAX) return MQ_ERR_SIZE;
    if (!al16(w_tiles) || !al16(y) || !al16(workspace) || ((uintptr_t)scale & 3u)) return MQ_ERR_ARG;
    size_t need = 0;
    mq_batch_matmul_workspace_bytes(K, &need);
    if (workspace_bytes < need) return MQ_ERR_SIZE;
    int dev = 0;
    cudaError_t e = setup_device(dev);
    if (e != cudaSuccess) return (int)e;
    uint8_t* ws = (uint8_t*)workspace;
    if ((e = cudaMemsetAsync(ws, 0, 256, stream)) != cudaSuccess) return (int)e;
    xpack_kernel<<<g_sms[dev], 256, 0, stream>>>(x, ws + 256, K, B, (unsigned*)ws);
    if ((e = cudaGetLastError()) != cudaSuccess) return (int)e;
    MMParams Q{};
    Q.w = w_tiles;
    Q.scale = scale;
    Q.xa = ws + 256;
    Q.y = y;
    Q.ctl = (unsigned*)ws;
    Q.budget_ns = 2000000000ull;
    Q.M = M;
    Q.K = K;
    Q.B = B;
    const int grid = g_sms[dev] < M / TROWS ? g_sms[dev] : M / TROWS;
    matmul_kernel<<<grid, NT, sizeof(Smem), stream>>>(Q);
    return (int)cudaGetLastError();
}

extern "C" int mq_batch_decode(const MQBatchArgs* a, int num_steps, cudaStream_t stream) {
    using namespace batch;
    if (!a || num_steps <= 0) return MQ_ERR_ARG;
    if (a->batch < 1 || a->batch > BMAX) return MQ_ERR_SIZE;
    if (a->num_layers < 1 || a->max_seq_len < 1) return MQ_ERR_ARG;
    if (a->max_seq_len > 32768) return MQ_ERR_SIZE;
    if (!a->embed_weight || !a->layer_weights || !a->scales || !a->final_norm_weight || !a->lm_head_weight ||
        !a->lm_head_scale || !a->cos_table || !a->sin_table || !a->k_cache || !a->v_cache || !a->tokens ||
        !a->positions || !a->workspace)
        return MQ_ERR_ARG;
    if (!al16(a->lm_head_weight) || !al16(a->k_cache) || !al16(a->v_cache) || !al16(a->workspace) ||
        !al16(a->embed_weight) || (a->logits && !al16(a->logits)))
        return MQ_ERR_ARG;
    const Layout Lw = layout(a->batch);
    if (a->workspace_bytes < Lw.total) return MQ_ERR_SIZE;
    int dev = 0;
    cudaError_t e = setup_device(dev);
    if (e != cudaSuccess) return (int)e;
    if (g_sms[dev] < MIN_SMS) return MQ_ERR_DEVICE;
    uint8_t* ws = (uint8_t*)a->workspace;
    Params P{};
    P.embed = (const __nv_bfloat16*)a->embed_weight;
    P.layers = a->layer_weights;
    P.scales = a->scales;
    P.final_norm = (const __nv_bfloat16*)a->final_norm_weight;
    P.lm_w = (const int8_t*)a->lm_head_weight;
    P.lm_scale = a->lm_head_scale;
    P.cos_t = (const __nv_bfloat16*)a->cos_table;
    P.sin_t = (const __nv_bfloat16*)a->sin_table;
    P.kc = (__nv_bfloat16*)a->k_cache;
    P.vc = (__nv_bfloat16*)a->v_cache;
    P.tokens_in = a->tokens;
    P.tokens_out = a->tokens;          // in place: token j+1 feeds step j+2
    P.positions = a->positions;
    P.h = (float*)(ws + Lw.h);
    P.act = (float*)(ws + Lw.act);
    P.qkv = (float*)(ws + Lw.qkv);
    P.xa_qkv = ws + Lw.xa_qkv;
    P.xa_o = ws + Lw.xa_o;
    P.xa_gu = ws + Lw.xa_gu;
    P.xa_dn = ws + Lw.xa_dn;
    P.ss_a = (float*)(ws + Lw.ss_a);
    P.ss_b = (float*)(ws + Lw.ss_b);
    P.part = (float*)(ws + Lw.part);
    P.best = (unsigned long long*)(ws + Lw.best);
    P.ctl = (unsigned*)(ws + Lw.ctl);
    P.logits = a->logits;
    P.trace = a->trace;
    P.budget_ns = a->wait_budget_ns ? a->wait_budget_ns : 2000000000ull;
    P.B = a->batch;
    P.L = a->num_layers;
    P.max_seq = a->max_seq_len;
    P.attn_scale = a->attn_scale;
    P.prefill = a->prefill;
    P.lm_tile0 = 0;
    P.lm_tiles = VOCAB / TROWS;
    P.keys_out = a->keys_out;
    if (a->vocab_shards > 1 || a->keys_out) {
        if (a->vocab_shards < 1 || a->vocab_shard < 0 || a->vocab_shard >= a->vocab_shards || !a->keys_out ||
            num_steps != 1 || a->prefill)
            return MQ_ERR_ARG;
        P.lm_tile0 = split_lo(VOCAB / TROWS, a->vocab_shards, a->vocab_shard);
        P.lm_tiles = split_lo(VOCAB / TROWS, a->vocab_shards, a->vocab_shard + 1) - P.lm_tile0;
    }
    if (P.prefill && num_steps != 1) return MQ_ERR_ARG;
    {
        // the tensor maps and the kernel's row index address cache rows with 32-bit integers
        const long long rows_ll = (long long)(a->prefill ? 1 : a->batch) * a->num_layers * NKVH * a->max_seq_len;
        if (rows_ll + ACH > 0x7fffffffLL) return MQ_ERR_SIZE;
        const int cache_rows = (int)rows_ll;
        if ((e = encode_cache_map(&P.tm_k, a->k_cache, cache_rows)) != cudaSuccess) return (int)e;
        if ((e = encode_cache_map(&P.tm_v, a->v_cache, cache_rows)) != cudaSuccess) return (int)e;
    }
    void* args[] = {&P};
    for (int j = 0; j < num_steps; ++j) {
        e = cudaLaunchCooperativeKernel((const void*)batch_kernel, dim3(g_sms[dev]), dim3(NT), args, sizeof(Smem) + 1024, stream);
        if (e != cudaSuccess) return (int)e;
    }
    return 0;
}

extern "C" int mq_batch_status(const void* workspace, int* code, int* info) {
    if (!workspace || !code || !info) return MQ_ERR_ARG;
    unsigned h[4] = {0, 0, 0, 0};
    cudaError_t e = cudaMemcpy(h, workspace, sizeof(h), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return (int)e;
    *code = (int)h[2];
    *info = (int)h[3];
    return 0;
}
