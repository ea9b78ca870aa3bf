// batch_kernel.cu -- batched greedy decode of Qwen3-0.6B on B200 (sm_100a):
// B independent sequences (each at its own position, with its own KV cache)
// advance one token per launch, sharing one pass over the INT8 weights.
//
// Per layer six phases separated by bounded grid barriers (a batched step is
// KV-bound, ~1 ms, so ~1.2 us per barrier is affordable and all data can move
// through plain global buffers):
//   QKV   X = bf16(RMSNorm(h)) staged in shared memory; weight-stationary GEMM
//         on the tensor cores (mma.sync m16n8k16 bf16): INT8 weight rows are
//         dequantised to bf16 exactly in registers, the per-row scale is
//         applied in the epilogue  -> qkv[b][4096] fp32
//   ATTN  one warp per (sequence, KV head, 256-position split): QK-RMSNorm +
//         RoPE at the sequence's own position, K/V write, flash-decode over
//         the cached positions (KV chunks bulk-copied into the warp's shared
//         buffer)  -> split partials (m, l, acc)
//   MERGE one warp per (sequence, q head): merges the splits -> attn bf16
//   O     GEMM + residual -> act fp32
//   GU    X = bf16(RMSNorm(act)); gate and up GEMM, SiLU(gate)*up -> mlp bf16
//   DOWN  GEMM + residual -> h (rounded to bf16, as between layers of the
//         batch-1 kernel)
// then RMSNorm + LM-head GEMM with a per-sequence packed argmax.
// Activations enter the tensor cores as two bf16 parts, x = hi + lo (about 16
// significant bits), each multiplied by the exactly dequantised bf16 weights
// with fp32 accumulation.
#include "common.cuh"
#include <stdlib.h>

namespace mq {
namespace batch {

constexpr int BMAX = 64;                 // sequences per launch (8 mma n-tiles)
constexpr int NW = 12;                   // warps per CTA
constexpr int NT = NW * 32;
constexpr int SLAB = 512;                // k columns staged at a time
constexpr int XS_STRIDE = SLAB + 8;      // bf16 elements per staged activation row (16-byte skew)
constexpr int SPLIT_POS = 256;           // attention positions per warp item
constexpr int MAX_SPLITS_B = 128;        // per sequence: max_seq <= 32768
constexpr int PARTW = 2 * HD + 4;        // acc[2][128], m[2], l[2]
constexpr int GROUP_ROWS = 32;           // weight rows staged per GEMM group (K = 1024)

struct Params {
    // weights (padded rows: stride = row bytes + ROW_SKEW)
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
    float* h;                   // [B][1024]
    float* act;                 // [B][1024]
    float* qkv;                 // [B][4096]
    float* attn;                // [B][2048]
    float* mlp;                 // [B][3072]
    float* part;                // [B][8][MAX_SPLITS_B][PARTW]
    unsigned long long* best;   // [B]
    unsigned int* ctl;          // [0] barrier counter, [1] exit counter, [2] error code, [3] error info
    float* logits;              // optional [B][VOCAB]
    unsigned long long* trace;  // optional [gridDim.x][8 * (L + 1)] globaltimer stamps
    unsigned long long budget_ns;
    int B, L, max_seq;
    float attn_scale;
};

// ---------------------------------------------------------------------------
// Shared memory (phases use disjoint views of one buffer)
// ---------------------------------------------------------------------------
struct GemmSmem {
    alignas(16) __nv_bfloat16 xs[2 * BMAX * XS_STRIDE];  // hi and lo planes, viewed as [2][ntok][width + 8], 133 KB
    alignas(16) uint8_t w[2][GROUP_ROWS * (HIDDEN + ROW_SKEW)];        // 2 x 33 KB
};
struct AttnSmem {
    alignas(16) uint8_t kv[NW][2 * 32 * HD * 2];   // per warp: 32 positions of K then V (16 KB)
    alignas(16) float q[NW][2][HD];
};
struct Smem {
    union {
        GemmSmem g;
        AttnSmem a;
    };
    uint64_t wbar[2];        // weight-group copies (outside the union: phases overwrite it)
    uint64_t abar[NW];       // per-warp KV chunk copies
    unsigned long long tokbest[BMAX];
    float rstd[BMAX];        // per-sequence RMSNorm factor of the phase being staged
    float red[NW];
    int abort_flag;
};

struct Ctx {
    Smem* sm;
    const Params* P;
    unsigned int barriers;   // grid barriers passed in this launch
};

__device__ __forceinline__ bool aborted(Ctx& c) {
    if (*(volatile int*)&c.sm->abort_flag) return true;
    if (ld_relaxed32(&c.P->ctl[2]) != 0) { *(volatile int*)&c.sm->abort_flag = 1; return true; }
    return false;
}
__device__ __noinline__ void fail(Ctx& c, int code, int info) {
    if (atomicCAS(&c.P->ctl[2], 0u, (unsigned)code) == 0u) atomicExch(&c.P->ctl[3], (unsigned)info);
    *(volatile int*)&c.sm->abort_flag = 1;
}

// Bounded grid barrier (release/acquire on a monotone counter reset per launch).
// Returns false when any CTA has failed; the caller then leaves the step.
__device__ __forceinline__ void stamp(const Ctx& c, int slot) {
    if (c.P->trace && threadIdx.x == 0)
        c.P->trace[(size_t)blockIdx.x * 8 * (c.P->L + 1) + slot] = globaltimer();
}

__device__ bool grid_barrier(Ctx& c, int where) {
    // Shared-memory bytes written through the generic proxy in this phase may be
    // overwritten by bulk copies (async proxy) in the next one.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    bool ok = !*(volatile int*)&c.sm->abort_flag;
    if (threadIdx.x == 0) {
        ++c.barriers;
        const unsigned target = c.barriers * gridDim.x;
        __threadfence();
        atomicAdd(&c.P->ctl[0], 1u);
        unsigned long long t0 = globaltimer();
        for (uint32_t it = 0;; ++it) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(&c.P->ctl[0]) : "memory");
            if ((int)(v - target) >= 0) break;
            if ((it & 63) == 63) {
                if (ld_relaxed32(&c.P->ctl[2]) != 0) { c.sm->abort_flag = 1; break; }
                if (globaltimer() - t0 > c.P->budget_ns) { fail(c, MQ_DEV_TIMEOUT_EXCHANGE, where); break; }
            }
        }
    } else {
        ++c.barriers;
    }
    __syncthreads();
    return ok && !*(volatile int*)&c.sm->abort_flag;
}


// ---------------------------------------------------------------------------
// Tensor-core GEMM pieces: D[16 rows x 8 tokens] += W[16 x 16] * X^T[16 x 8]
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t i8x2_to_bf16x2(uint32_t v) {  // two signed bytes -> two bf16 (exact)
    const float lo = (float)(int8_t)(v & 0xffu), hi = (float)(int8_t)((v >> 8) & 0xffu);
    __nv_bfloat162 r = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// A fragment of rows (ra, ra + 8) x k [k0, k0 + 16) from int8 rows in shared memory.
__device__ __forceinline__ void load_a(uint32_t (&a)[4], const uint8_t* ra, const uint8_t* rb, int k0, int t) {
    const uint16_t* pa = reinterpret_cast<const uint16_t*>(ra + k0 + 2 * t);
    const uint16_t* pb = reinterpret_cast<const uint16_t*>(rb + k0 + 2 * t);
    a[0] = i8x2_to_bf16x2(pa[0]);
    a[1] = i8x2_to_bf16x2(pb[0]);
    a[2] = i8x2_to_bf16x2(pa[4]);
    a[3] = i8x2_to_bf16x2(pb[4]);
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ bool mbar_wait_b(Ctx& c, uint64_t* bar, uint32_t parity, int where) {
    if (mbar_test(bar, parity)) return true;
    unsigned long long t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_test(bar, parity)) return true;
        if ((it & 63) == 0) {
            if (aborted(c)) return false;
            if (globaltimer() - t0 > c.P->budget_ns) { fail(c, MQ_DEV_TIMEOUT_RING, where); return false; }
        }
    }
}

// Writes 16 consecutive values (this lane's part of a 512-wide slab row) as hi/lo.
// Staged activations: xs viewed as [2][ntok][width + 8] (plane 0 = hi, 1 = lo).
template <int NTOK, int WIDTH>
struct XView {
    static constexpr int RS = WIDTH + 8;
    static constexpr int PS = NTOK * RS;
    static_assert(2 * PS <= 2 * BMAX * XS_STRIDE, "view exceeds the staging buffer");
};
template <int NTOK, int WIDTH>
__device__ __forceinline__ void put16(Smem* sm, int b, int k0, const float (&v)[16]) {
    using V = XView<NTOK, WIDTH>;
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
        const __nv_bfloat162 hi = __floats2bfloat162_rn(v[i], v[i + 1]);
        const float2 hf = __bfloat1622float2(hi);
        const __nv_bfloat162 lo = __floats2bfloat162_rn(v[i] - hf.x, v[i + 1] - hf.y);
        *reinterpret_cast<__nv_bfloat162*>(&sm->g.xs[b * V::RS + k0 + i]) = hi;
        *reinterpret_cast<__nv_bfloat162*>(&sm->g.xs[V::PS + b * V::RS + k0 + i]) = lo;
    }
}

// Loads 16 fp32 values [k0, k0 + 16) of a row (4 x float4, all issued together).
__device__ __forceinline__ void load16(const float* row, int k0, float (&v)[16]) {
    const float4* r = reinterpret_cast<const float4*>(row + k0);
    float4 q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = __ldcg(r + i);
#pragma unroll
    for (int i = 0; i < 4; ++i) { v[4 * i] = q[i].x; v[4 * i + 1] = q[i].y; v[4 * i + 2] = q[i].z; v[4 * i + 3] = q[i].w; }
}
__device__ __forceinline__ void load16_bf16(const __nv_bfloat16* row, int k0, float (&v)[16]) {
    const uint4* r = reinterpret_cast<const uint4*>(row + k0);
    const uint4 a = __ldg(r), b = __ldg(r + 1);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) { v[2 * i] = bf16_bits_to_f32(w[i] & 0xffffu); v[2 * i + 1] = bf16_bits_to_f32(w[i] >> 16); }
}

// Stages slab s (columns [s*SLAB, (s+1)*SLAB)) of X = RMSNorm(row_b) * w for the
// B sequences (rows >= B are zero); row(b) is the fp32 row of sequence b, or the
// bf16 embedding row when emb is set.  rstd is computed at s == 0 and kept in
// shared memory.  Lane l owns columns [16l, 16l + 16) of the slab.
template <bool EMB, class Row>
__device__ __forceinline__ void stage_norm_slab(Smem* sm, int B, int s, const __nv_bfloat16* w, Row row) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (s == 0) {
        for (int b = warp; b < B; b += NW) {
            float v0[16], v1[16];
            if constexpr (EMB) { load16_bf16(row(b), 16 * lane, v0); load16_bf16(row(b), 512 + 16 * lane, v1); }
            else { load16(row(b), 16 * lane, v0); load16(row(b), 512 + 16 * lane, v1); }
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) ss += v0[i] * v0[i] + v1[i] * v1[i];
            ss = warp_sum(ss);
            if (lane == 0) sm->rstd[b] = rsqrtf(ss / (float)HIDDEN + RMS_EPS);
        }
        __syncthreads();
    }
    float wv[16];
    load16_bf16(w, s * SLAB + 16 * lane, wv);
    for (int b = warp; b < BMAX; b += NW) {
        float v[16];
        if (b < B) {
            if constexpr (EMB) load16_bf16(row(b), s * SLAB + 16 * lane, v);
            else load16(row(b), s * SLAB + 16 * lane, v);
            const float r = sm->rstd[b];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = v[i] * r * wv[i];
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
        }
        put16<BMAX, SLAB>(sm, b, 16 * lane, v);
    }
}

// LM head: X = RMSNorm(h[n0 + i]) * w for 32 tokens, full width (lane owns
// columns [32 lane, 32 lane + 32)).
__device__ __forceinline__ void stage_norm_half(Smem* sm, int B, int n0, const float* h, const __nv_bfloat16* w) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float w0[16], w1[16];
    load16_bf16(w, 32 * lane, w0);
    load16_bf16(w, 32 * lane + 16, w1);
    for (int i = warp; i < 32; i += NW) {
        const int b = n0 + i;
        float v0[16], v1[16];
        if (b < B) {
            load16(h + (size_t)b * HIDDEN, 32 * lane, v0);
            load16(h + (size_t)b * HIDDEN, 32 * lane + 16, v1);
            float ss = 0.f;
#pragma unroll
            for (int k = 0; k < 16; ++k) ss += v0[k] * v0[k] + v1[k] * v1[k];
            ss = warp_sum(ss);
            const float r = rsqrtf(ss / (float)HIDDEN + RMS_EPS);
#pragma unroll
            for (int k = 0; k < 16; ++k) { v0[k] *= r * w0[k]; v1[k] *= r * w1[k]; }
        } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) v0[k] = v1[k] = 0.f;
        }
        put16<32, HIDDEN>(sm, i, 32 * lane, v0);
        put16<32, HIDDEN>(sm, i, 32 * lane + 16, v1);
    }
}

// Stages slab s of an fp32 [B][K] global matrix.
__device__ __forceinline__ void stage_copy(Smem* sm, int B, const float* src, int K, int s) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int b = warp; b < BMAX; b += NW) {
        float v[16];
        if (b < B) load16(src + (size_t)b * K, s * SLAB + 16 * lane, v);
        else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
        }
        put16<BMAX, SLAB>(sm, b, 16 * lane, v);
    }
}

// Issues the bulk copy of `n` padded rows (stride rs) starting at src into w
// buffer `buf`; thread 0 only.  Returns the bytes expected.
__device__ __forceinline__ void load_rows(Smem* sm, int buf, const uint8_t* src, int n, int rs, int dst_row) {
    uint8_t* dst = sm->g.w[buf] + (size_t)dst_row * rs;
    bulk_g2s(dst, src, (uint32_t)(n * rs), &sm->wbar[buf]);
}

// One GEMM group already being copied into w[buf]: NS = K/1024 slabs, staged by
// stage(s).  SETS = 1: plain rows (tile i = smem rows 16i..16i+15); SETS = 2:
// gate/up (tile i: gate rows at smem 32i.., up rows at 32i+16..), two
// accumulators per unit.  epi(row_in_group, token, value[SETS]).
template <int K, int SETS, int NTOK = BMAX, int WIDTH = SLAB, class Stage, class Epi>
__device__ bool gemm_group(Ctx& c, int buf, uint32_t& wuse, int rows, Stage stage, Epi epi) {
    constexpr int NS = K / WIDTH;
    constexpr int RS = K + ROW_SKEW;
    constexpr int NJ = NTOK / 8;      // n-tiles
    using V = XView<NTOK, WIDTH>;
    Smem* sm = c.sm;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int T = (rows + 15) / 16;
    const int nunits = T * NJ;   // <= 16 for every group here
    // four independent accumulation chains per unit and set: (hi, lo) x (even, odd k-step)
    float acc[2][SETS][4][4];
#pragma unroll
    for (int k = 0; k < 2; ++k)
#pragma unroll
        for (int q = 0; q < SETS; ++q)
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) acc[k][q][ch][0] = acc[k][q][ch][1] = acc[k][q][ch][2] = acc[k][q][ch][3] = 0.f;
    bool ok = true;
    for (int s = 0; s < NS; ++s) {
        if (s > 0) __syncthreads();
        stage(s);
        __syncthreads();
        if (s == 0) {
            ok = mbar_wait_b(c, &sm->wbar[buf], wuse & 1, 200 + buf);
            ++wuse;
        }
        const uint8_t* w = sm->g.w[buf];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int u = warp + k * NW;
            if (u >= nunits) continue;
            const int tile = u / NJ, j = u % NJ;
            const __nv_bfloat16* xh = sm->g.xs + (j * 8 + g) * V::RS;
            const __nv_bfloat16* xl = xh + V::PS;
#pragma unroll
            for (int q = 0; q < SETS; ++q) {
                const int base = SETS == 1 ? tile * 16 : tile * 32 + q * 16;
                const int lim = SETS == 1 ? rows - 1 : base + 15;
                const uint8_t* ra = w + (size_t)min(base + g, lim) * RS + (size_t)s * WIDTH;
                const uint8_t* rb = w + (size_t)min(base + g + 8, lim) * RS + (size_t)s * WIDTH;
#pragma unroll 2
                for (int ks = 0; ks < WIDTH / 16; ks += 2) {
                    uint32_t a0[4], a1[4];
                    load_a(a0, ra, rb, ks * 16, t);
                    load_a(a1, ra, rb, ks * 16 + 16, t);
                    const int k0 = ks * 16 + 2 * t;
                    mma_bf16(acc[k][q][0], a0, *reinterpret_cast<const uint32_t*>(xh + k0), *reinterpret_cast<const uint32_t*>(xh + k0 + 8));
                    mma_bf16(acc[k][q][1], a0, *reinterpret_cast<const uint32_t*>(xl + k0), *reinterpret_cast<const uint32_t*>(xl + k0 + 8));
                    mma_bf16(acc[k][q][2], a1, *reinterpret_cast<const uint32_t*>(xh + k0 + 16), *reinterpret_cast<const uint32_t*>(xh + k0 + 24));
                    mma_bf16(acc[k][q][3], a1, *reinterpret_cast<const uint32_t*>(xl + k0 + 16), *reinterpret_cast<const uint32_t*>(xl + k0 + 24));
                }
            }
        }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int u = warp + k * NW;
        if (u >= nunits) continue;
        const int tile = u / NJ, j = u % NJ;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int r = tile * 16 + g + (e >= 2 ? 8 : 0);
            const int n = j * 8 + 2 * t + (e & 1);
            float v[SETS];
#pragma unroll
            for (int q = 0; q < SETS; ++q)
                v[q] = (acc[k][q][0][e] + acc[k][q][1][e]) + (acc[k][q][2][e] + acc[k][q][3][e]);
            if (r < rows) epi(r, n, v);
        }
    }
    __syncthreads();
    return ok;
}

// Copies rows [a, a + n) (padded, stride rs) of the matrix at base into w[buf]
// at smem row dst_row; thread 0 only, after arming the barrier.
__device__ __forceinline__ void copy_rows(Smem* sm, int buf, const void* base, int a, int n, int rs, int dst_row) {
    if (n <= 0) return;
    bulk_g2s(sm->g.w[buf] + (size_t)dst_row * rs, (const uint8_t*)base + (size_t)a * rs, (uint32_t)(n * rs),
             &sm->wbar[buf]);
}

// ---------------------------------------------------------------------------
// Attention: one warp per (sequence, KV head, split)
// ---------------------------------------------------------------------------
__device__ __forceinline__ int nsplit_of(int pos) { return pos / SPLIT_POS + 1; }  // cache_len = pos + 1

__device__ void attn_item(Ctx& c, const Params& P, int l, int b, int kvh, int s, uint32_t& ause) {
    Smem* sm = c.sm;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = P.positions[b];
    const int c_len = pos + 1;
    const int p0 = s * SPLIT_POS;
    const bool owner = p0 + SPLIT_POS >= c_len;   // the split that holds the current position
    const int p1 = owner ? pos : p0 + SPLIT_POS;  // cached positions [p0, p1)
    const LayerWeights& w = P.layers[l];
    const float* qkv = P.qkv + (size_t)b * QKV_ROWS;
    const __nv_bfloat16* cosr = P.cos_t + (size_t)pos * HD;
    const __nv_bfloat16* sinr = P.sin_t + (size_t)pos * HD;
    float* q = sm->a.q[warp][0];
    // QK-RMSNorm + split-half RoPE (lane holds dims lane + 32j; partners j, j + 2)
    auto norm_rope = [&](const float* raw, const __nv_bfloat16* nw, float out[4]) {
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
    };
#pragma unroll
    for (int hq = 0; hq < 2; ++hq) {
        float o[4];
        norm_rope(qkv + (2 * kvh + hq) * HD, (const __nv_bfloat16*)w.q_norm_weight, o);
#pragma unroll
        for (int j = 0; j < 4; ++j) q[hq * HD + lane + 32 * j] = o[j];
    }
    uint16_t kcur[4], vcur[4];
    if (owner) {
        float o[4];
        norm_rope(qkv + QSZ + kvh * HD, (const __nv_bfloat16*)w.k_norm_weight, o);
        const size_t off = ((((size_t)b * P.L + l) * NKVH + kvh) * (size_t)P.max_seq + pos) * HD;
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
    const float4* q0v = reinterpret_cast<const float4*>(q);
    const float4* q1v = reinterpret_cast<const float4*>(q + HD);
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
    const float scale = P.attn_scale;
    uint8_t* buf = sm->a.kv[warp];
    const uint16_t* kb = reinterpret_cast<const uint16_t*>(buf);
    const uint16_t* vb = reinterpret_cast<const uint16_t*>(buf + 32 * HD * 2);
    auto chunk = [&](int n) {
        float s0 = -INFINITY, s1 = -INFINITY;
        if (lane < n) {
            const uint16_t* kr = kb + lane * HD;
            float x0 = 0.f, x1 = 0.f, y0 = 0.f, y1 = 0.f;
#pragma unroll 8
            for (int i = 0; i < HD / 4; ++i) {
                const int d4 = (lane + i) & (HD / 4 - 1);
                const uint2 kw = *reinterpret_cast<const uint2*>(kr + 4 * d4);
                const float k0 = bf16_bits_to_f32(kw.x & 0xffffu), k1 = bf16_bits_to_f32(kw.x >> 16);
                const float k2 = bf16_bits_to_f32(kw.y & 0xffffu), k3 = bf16_bits_to_f32(kw.y >> 16);
                const float4 qa = q0v[d4], qb = q1v[d4];
                x0 = fmaf(qa.x, k0, x0); x1 = fmaf(qa.y, k1, x1); x0 = fmaf(qa.z, k2, x0); x1 = fmaf(qa.w, k3, x1);
                y0 = fmaf(qb.x, k0, y0); y1 = fmaf(qb.y, k1, y1); y0 = fmaf(qb.z, k2, y0); y1 = fmaf(qb.w, k3, y1);
            }
            s0 = (x0 + x1) * scale;
            s1 = (y0 + y1) * scale;
        }
        const float n0 = fmaxf(m0, warp_max(s0)), n1 = fmaxf(m1, warp_max(s1));
        const float c0 = expf(m0 - n0), c1 = expf(m1 - n1);
        const float e0 = lane < n ? expf(s0 - n0) : 0.f;
        const float e1 = lane < n ? expf(s1 - n1) : 0.f;
        l0 = l0 * c0 + warp_sum(e0);
        l1 = l1 * c1 + warp_sum(e1);
#pragma unroll
        for (int j = 0; j < 4; ++j) { a0[j] *= c0; a1[j] *= c1; }
        for (int p = 0; p < n; ++p) {
            const float ep0 = __shfl_sync(0xffffffffu, e0, p), ep1 = __shfl_sync(0xffffffffu, e1, p);
            const uint2 vw = *reinterpret_cast<const uint2*>(vb + p * HD + 4 * lane);
            const float v0 = bf16_bits_to_f32(vw.x & 0xffffu), v1 = bf16_bits_to_f32(vw.x >> 16);
            const float v2 = bf16_bits_to_f32(vw.y & 0xffffu), v3 = bf16_bits_to_f32(vw.y >> 16);
            a0[0] = fmaf(ep0, v0, a0[0]); a0[1] = fmaf(ep0, v1, a0[1]); a0[2] = fmaf(ep0, v2, a0[2]); a0[3] = fmaf(ep0, v3, a0[3]);
            a1[0] = fmaf(ep1, v0, a1[0]); a1[1] = fmaf(ep1, v1, a1[1]); a1[2] = fmaf(ep1, v2, a1[2]); a1[3] = fmaf(ep1, v3, a1[3]);
        }
        m0 = n0;
        m1 = n1;
    };
    const size_t head = (((size_t)b * P.L + l) * NKVH + kvh) * (size_t)P.max_seq * HD;
    for (int p = p0; p < p1; p += 32) {
        const int n = min(32, p1 - p);
        __syncwarp();
        if (lane == 0) {
            fence_proxy_async();
            mbar_arrive_expect_tx(&sm->abar[warp], 2u * n * HD * 2);
            bulk_g2s(buf, P.kc + head + (size_t)p * HD, n * HD * 2, &sm->abar[warp]);
            bulk_g2s(buf + 32 * HD * 2, P.vc + head + (size_t)p * HD, n * HD * 2, &sm->abar[warp]);
        }
        const bool okw = mbar_wait_b(c, &sm->abar[warp], ause & 1, 300);
        ++ause;
        if (!okw) return;
        chunk(n);
    }
    if (owner) {  // the current position from registers
        __syncwarp();
        uint16_t* kw = reinterpret_cast<uint16_t*>(buf);
        uint16_t* vw = reinterpret_cast<uint16_t*>(buf + 32 * HD * 2);
#pragma unroll
        for (int j = 0; j < 4; ++j) { kw[lane + 32 * j] = kcur[j]; vw[lane + 32 * j] = vcur[j]; }
        __syncwarp();
        chunk(1);
    }
    float* out = P.part + (((size_t)b * NKVH + kvh) * MAX_SPLITS_B + s) * PARTW;
    *reinterpret_cast<float4*>(out + 4 * lane) = make_float4(a0[0], a0[1], a0[2], a0[3]);
    *reinterpret_cast<float4*>(out + HD + 4 * lane) = make_float4(a1[0], a1[1], a1[2], a1[3]);
    if (lane == 0) { out[2 * HD] = m0; out[2 * HD + 1] = m1; out[2 * HD + 2] = l0; out[2 * HD + 3] = l1; }
}

// One warp per (sequence, q head): merge the splits into attn (bf16).
__device__ void merge_item(const Params& P, int b, int qh) {
    const int lane = threadIdx.x & 31;
    const int kvh = qh >> 1, hh = qh & 1;
    const int ns = nsplit_of(P.positions[b]);
    const float* base = P.part + ((size_t)b * NKVH + kvh) * MAX_SPLITS_B * PARTW;
    float M = -INFINITY;
    for (int s = 0; s < ns; ++s) M = fmaxf(M, __ldcg(base + (size_t)s * PARTW + 2 * HD + hh));
    float L = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < ns; ++s) {
        const float* ps = base + (size_t)s * PARTW;
        const float e = expf(__ldcg(ps + 2 * HD + hh) - M);
        L = fmaf(__ldcg(ps + 2 * HD + 2 + hh), e, L);
        const float4 a = __ldcg(reinterpret_cast<const float4*>(ps + hh * HD + 4 * lane));
        o[0] = fmaf(a.x, e, o[0]); o[1] = fmaf(a.y, e, o[1]); o[2] = fmaf(a.z, e, o[2]); o[3] = fmaf(a.w, e, o[3]);
    }
    const float inv = 1.f / L;
    float* dst = P.attn + (size_t)b * QSZ + qh * HD + 4 * lane;
    *reinterpret_cast<float4*>(dst) = make_float4(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv);
}


// ---------------------------------------------------------------------------
// The step kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT, 1) batch_kernel(const Params P) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem* sm = reinterpret_cast<Smem*>(smem_raw);
    Ctx c{sm, &P, 0u};
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = gridDim.x, cta = blockIdx.x;
    const int B = P.B;
    if (threadIdx.x == 0) {
        mbar_init(&sm->wbar[0], 1);
        mbar_init(&sm->wbar[1], 1);
        for (int i = 0; i < NW; ++i) mbar_init(&sm->abar[i], 1);
        sm->abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i < BMAX; i += NT) sm->tokbest[i] = 0ull;
    __syncthreads();
    // Every CTA validates the per-sequence inputs before touching memory with them.
    for (int t = threadIdx.x; t < B; t += NT) {
        const int tok = P.tokens_in[t], pos = P.positions[t];
        if (tok < 0 || tok >= VOCAB) fail(c, MQ_DEV_BAD_TOKEN, t);
        if (pos < 0 || pos >= P.max_seq) fail(c, MQ_DEV_BAD_POSITION, t);
    }
    __syncthreads();
    uint32_t wuse[2] = {0u, 0u};
    uint32_t ause = 0u;   // this warp's KV-chunk barrier uses
    bool ok = !*(volatile int*)&sm->abort_flag;
    for (int l = 0; l < P.L && ok; ++l) {
        const LayerWeights& w = P.layers[l];
        const ScalePointers& sc = P.scales[l];
        // ---- QKV ----
        {
            constexpr int RS = HIDDEN + ROW_SKEW;
            const int r0 = split_lo(QKV_ROWS, nb, cta), r1 = split_lo(QKV_ROWS, nb, cta + 1);
            if (threadIdx.x == 0) {
                fence_proxy_async();
                mbar_arrive_expect_tx(&sm->wbar[0], (uint32_t)((r1 - r0) * RS));
                int done = 0;
                while (done < r1 - r0) {
                    const int row = r0 + done;
                    const void* base; int first, lim;
                    if (row < QSZ) { base = w.q_proj_weight; first = 0; lim = QSZ; }
                    else if (row < QSZ + KVSZ) { base = w.k_proj_weight; first = QSZ; lim = QSZ + KVSZ; }
                    else { base = w.v_proj_weight; first = QSZ + KVSZ; lim = QKV_ROWS; }
                    const int m = min(r1 - r0 - done, lim - row);
                    copy_rows(sm, 0, base, row - first, m, RS, done);
                    done += m;
                }
            }
            auto stage = [&](int s_) {
                const __nv_bfloat16* nw = (const __nv_bfloat16*)w.input_layernorm_weight;
                if (l == 0) {
                    // h = embedding rows; CTA 0 also stores them as the fp32 residual.
                    auto row = [&](int b) { return P.embed + (size_t)P.tokens_in[b] * HIDDEN; };
                    stage_norm_slab<true>(sm, B, s_, nw, row);
                    if (cta == 0 && s_ == 0)
                        for (int i = threadIdx.x; i < B * HIDDEN; i += NT)
                            P.h[i] = __bfloat162float(P.embed[(size_t)P.tokens_in[i / HIDDEN] * HIDDEN + i % HIDDEN]);
                } else {
                    stage_norm_slab<false>(sm, B, s_, nw, [&](int b) { return (const float*)P.h + (size_t)b * HIDDEN; });
                }
            };
            const float* sq = sc.q_scale; const float* sk = sc.k_scale; const float* sv = sc.v_scale;
            ok = gemm_group<HIDDEN, 1>(c, 0, wuse[0], r1 - r0, stage, [&](int r, int n, const float* v) {
                if (n >= B) return;
                const int row = r0 + r;
                const float s_ = row < QSZ ? sq[row] : (row < QSZ + KVSZ ? sk[row - QSZ] : sv[row - QSZ - KVSZ]);
                P.qkv[(size_t)n * QKV_ROWS + row] = v[0] * s_;
            }) && ok;
        }
        stamp(c, l * 8 + 1);
        if (!grid_barrier(c, 1)) { ok = false; break; }
        // ---- attention ----
        {
            // items (b, kvh, s) enumerated sequence-major
            int item = cta * NW + warp;
            const int stride = nb * NW;
            int b = 0, base = 0;
            while (b < B) {
                const int cnt = NKVH * nsplit_of(P.positions[b]);
                while (item < base + cnt) {
                    const int r = item - base;
                    attn_item(c, P, l, b, r / nsplit_of(P.positions[b]), r % nsplit_of(P.positions[b]), ause);
                    item += stride;
                }
                base += cnt;
                ++b;
            }
        }
        stamp(c, l * 8 + 2);
        if (!grid_barrier(c, 2)) { ok = false; break; }
        // ---- merge ----
        for (int it = cta * NW + warp; it < B * NQH; it += nb * NW) merge_item(P, it / NQH, it % NQH);
        stamp(c, l * 8 + 3);
        if (!grid_barrier(c, 3)) { ok = false; break; }
        // ---- O + residual ----
        {
            constexpr int K = QSZ, RS = K + ROW_SKEW;
            const int r0 = split_lo(HIDDEN, nb, cta), r1 = split_lo(HIDDEN, nb, cta + 1);
            if (threadIdx.x == 0) {
                fence_proxy_async();
                mbar_arrive_expect_tx(&sm->wbar[1], (uint32_t)((r1 - r0) * RS));
                copy_rows(sm, 1, w.o_proj_weight, r0, r1 - r0, RS, 0);
            }
            const float* so = sc.o_scale;
            ok = gemm_group<K, 1>(c, 1, wuse[1], r1 - r0, [&](int s_) { stage_copy(sm, B, P.attn, K, s_); },
                                  [&](int r, int n, const float* v) {
                                      if (n >= B) return;
                                      const size_t i = (size_t)n * HIDDEN + r0 + r;
                                      P.act[i] = v[0] * so[r0 + r] + __ldcg(P.h + i);
                                  }) && ok;
        }
        stamp(c, l * 8 + 4);
        if (!grid_barrier(c, 4)) { ok = false; break; }
        // ---- gate/up + SiLU ----
        {
            constexpr int RS = HIDDEN + ROW_SKEW;
            const int p0 = split_lo(INTER, nb, cta), p1 = split_lo(INTER, nb, cta + 1);
            const float* sg = sc.gate_scale; const float* su = sc.up_scale;
            for (int gp = p0, gi = 0; gp < p1 && ok; gp += 16, ++gi) {
                const int np = min(16, p1 - gp);
                const int buf = gi & 1;
                if (threadIdx.x == 0) {
                    fence_proxy_async();
                    mbar_arrive_expect_tx(&sm->wbar[buf], (uint32_t)(2 * np * RS));
                    copy_rows(sm, buf, w.gate_proj_weight, gp, np, RS, 0);
                    copy_rows(sm, buf, w.up_proj_weight, gp, np, RS, 16);
                }
                ok = gemm_group<HIDDEN, 2>(c, buf, wuse[buf], np,
                                           [&](int s_) {
                                               stage_norm_slab<false>(sm, B, s_, (const __nv_bfloat16*)w.post_attn_layernorm_weight,
                                                                      [&](int b) { return (const float*)P.act + (size_t)b * HIDDEN; });
                                           },
                                           [&](int r, int n, const float* v) {
                                               if (n >= B) return;
                                               const int row = gp + r;
                                               const float gd = v[0] * sg[row], ud = v[1] * su[row];
                                               const float silu = gd / (1.0f + expf(-gd));
                                               P.mlp[(size_t)n * INTER + row] = silu * ud;
                                           }) && ok;
            }
        }
        stamp(c, l * 8 + 5);
        if (!grid_barrier(c, 5)) { ok = false; break; }
        // ---- down + residual -> h ----
        {
            constexpr int K = INTER, RS = K + ROW_SKEW;
            const int r0 = split_lo(HIDDEN, nb, cta), r1 = split_lo(HIDDEN, nb, cta + 1);
            if (threadIdx.x == 0) {
                fence_proxy_async();
                mbar_arrive_expect_tx(&sm->wbar[0], (uint32_t)((r1 - r0) * RS));
                copy_rows(sm, 0, w.down_proj_weight, r0, r1 - r0, RS, 0);
            }
            const float* sd = sc.down_scale;
            ok = gemm_group<K, 1>(c, 0, wuse[0], r1 - r0, [&](int s_) { stage_copy(sm, B, P.mlp, K, s_); },
                                  [&](int r, int n, const float* v) {
                                      if (n >= B) return;
                                      const size_t i = (size_t)n * HIDDEN + r0 + r;
                                      P.h[i] = __bfloat162float(__float2bfloat16_rn(v[0] * sd[r0 + r] + __ldcg(P.act + i)));
                                  }) && ok;
        }
        stamp(c, l * 8 + 6);
        if (!grid_barrier(c, 6)) { ok = false; break; }
    }
    // ---- final norm + LM head + per-sequence argmax ----
    // Two halves of 32 sequences: each half's normalised activations are staged
    // once at full width and all of this CTA's LM-head rows stream past them.
    if (ok) {
        constexpr int RS = HIDDEN + ROW_SKEW;
        const int r0 = split_lo(VOCAB, nb, cta), r1 = split_lo(VOCAB, nb, cta + 1);
        auto issue = [&](int gr0, int buf) {
            const int n = min(GROUP_ROWS, r1 - gr0);
            fence_proxy_async();
            mbar_arrive_expect_tx(&sm->wbar[buf], (uint32_t)(n * RS));
            copy_rows(sm, buf, P.lm_w, gr0, n, RS, 0);
        };
        const int halves = (B + 31) / 32;
        int gi = 0;
        for (int hf = 0; hf < halves && ok; ++hf) {
            const int n0 = hf * 32;
            if (threadIdx.x == 0) issue(r0, gi & 1);
            for (int gr = r0; gr < r1 && ok; gr += GROUP_ROWS, ++gi) {
                const int buf = gi & 1;
                const int n = min(GROUP_ROWS, r1 - gr);
                // the other buffer was released by the previous group's trailing barrier
                if (threadIdx.x == 0 && gr + GROUP_ROWS < r1) issue(gr + GROUP_ROWS, buf ^ 1);
                const bool first = gr == r0;
                ok = gemm_group<HIDDEN, 1, 32, HIDDEN>(
                         c, buf, wuse[buf], n,
                         [&](int) { if (first) stage_norm_half(sm, B, n0, P.h, P.final_norm); },
                         [&](int r, int tl, const float* v) {
                             const int tok = n0 + tl;
                             if (tok >= B) return;
                             const int row = gr + r;
                             const float lg = v[0] * P.lm_scale[row];
                             if (P.logits) P.logits[(size_t)tok * VOCAB + row] = lg;
                             const unsigned long long key =
                                 (((unsigned long long)float_order_key(lg)) << 32) | (uint32_t)(~(uint32_t)row);
                             atomicMax(&sm->tokbest[tok], key);
                         }) && ok;
            }
        }
        __syncthreads();
        for (int t = threadIdx.x; t < B; t += NT) atomicMax(&P.best[t], sm->tokbest[t]);
    }
    stamp(c, P.L * 8 + 6);
    grid_barrier(c, 7);
    stamp(c, P.L * 8 + 7);
    if (cta == 0) {
        const bool err = ld_relaxed32(&P.ctl[2]) != 0;
        for (int t = threadIdx.x; t < B; t += NT) {
            const unsigned long long k = __ldcg(P.best + t);
            P.tokens_out[t] = (err || k == 0ull) ? -1 : (int)(~(uint32_t)k);
            P.best[t] = 0ull;
            if (!err) P.positions[t] += 1;
        }
    }
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
    (void)lane;
}


// ===========================================================================
// Host side
// ===========================================================================
namespace {
struct Layout {
    size_t h, act, qkv, attn, mlp, part, best, ctl, total;
};
size_t up256(size_t x) { return (x + 255) & ~(size_t)255; }
Layout layout(int B) {
    Layout L{};
    size_t o = 0;
    L.ctl = o;  o += up256(4 * sizeof(unsigned));
    L.best = o; o += up256((size_t)B * sizeof(unsigned long long));
    L.h = o;    o += up256((size_t)B * HIDDEN * 4);
    L.act = o;  o += up256((size_t)B * HIDDEN * 4);
    L.qkv = o;  o += up256((size_t)B * QKV_ROWS * 4);
    L.attn = o; o += up256((size_t)B * QSZ * 4);
    L.mlp = o;  o += up256((size_t)B * INTER * 4);
    L.part = o; o += up256((size_t)B * NKVH * MAX_SPLITS_B * PARTW * 4);
    L.total = o;
    return L;
}
constexpr int MAX_DEV = 64;
bool g_attr[MAX_DEV];
int g_sms[MAX_DEV];
bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }
}  // namespace
}  // namespace batch
}  // namespace mq

using namespace mq;

extern "C" int mq_batch_workspace_bytes(int batch, size_t* bytes) {
    if (batch < 1 || batch > batch::BMAX || !bytes) return MQ_ERR_ARG;
    *bytes = batch::layout(batch).total;
    return 0;
}

extern "C" int mq_batch_decode(const MQBatchArgs* a, int num_steps, cudaStream_t stream) {
    using namespace batch;
    if (!a || num_steps <= 0) return MQ_ERR_ARG;
    if (a->batch < 1 || a->batch > BMAX) return MQ_ERR_SIZE;
    if (a->num_layers < 1 || a->max_seq_len < 1) return MQ_ERR_ARG;
    if (a->max_seq_len > MAX_SPLITS_B * SPLIT_POS) return MQ_ERR_SIZE;
    if (!a->embed_weight || !a->layer_weights || !a->scales || !a->final_norm_weight || !a->lm_head_weight ||
        !a->lm_head_scale || !a->cos_table || !a->sin_table || !a->k_cache || !a->v_cache || !a->tokens ||
        !a->positions || !a->workspace)
        return MQ_ERR_ARG;
    if (!al16(a->lm_head_weight) || !al16(a->k_cache) || !al16(a->v_cache) || !al16(a->workspace)) return MQ_ERR_ARG;
    const Layout Lw = layout(a->batch);
    if (a->workspace_bytes < Lw.total) return MQ_ERR_SIZE;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= MAX_DEV) return MQ_ERR_DEVICE;
    if (!g_attr[dev]) {
        if ((e = cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return (int)e;
        if ((e = cudaFuncSetAttribute(batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem))) !=
            cudaSuccess)
            return (int)e;
        g_attr[dev] = true;
    }
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
    P.attn = (float*)(ws + Lw.attn);
    P.mlp = (float*)(ws + Lw.mlp);
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
    void* args[] = {&P};
    for (int j = 0; j < num_steps; ++j) {
        e = cudaLaunchCooperativeKernel((const void*)batch_kernel, dim3(g_sms[dev]), dim3(NT), args, sizeof(Smem), stream);
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
