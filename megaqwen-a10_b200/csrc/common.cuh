// common.cuh -- shapes, launch geometry and device primitives shared by the
// sm_100a kernels of this library.
//
// Model shapes are the Qwen3-0.6B constants of the reference's config.cuh:30-40.
// The launch geometry is B200-specific: one persistent CTA per SM (148 on B200),
// NCW consumer warps plus one producer warp that streams weights and KV rows
// into a shared-memory ring with cp.async.bulk (non-multicast, local HBM only).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include "../../include/megaqwen_b200.h"

namespace mq {

constexpr int HIDDEN = 1024;
constexpr int INTER = 3072;
constexpr int NQH = 16;
constexpr int NKVH = 8;
constexpr int HD = 128;
constexpr int QSZ = NQH * HD;        // 2048
constexpr int KVSZ = NKVH * HD;      // 1024
constexpr int QKV_ROWS = QSZ + 2 * KVSZ;  // 4096
constexpr int VOCAB = 151936;
constexpr float RMS_EPS = 1e-6f;

#ifndef MQ_NCW
#define MQ_NCW 12
#endif
#ifndef MQ_STAGE_BYTES
#define MQ_STAGE_BYTES 16640
#endif
#ifndef MQ_NSTAGE
#define MQ_NSTAGE 10
#endif
constexpr int NCW = MQ_NCW;                   // consumer warps
constexpr int NCT = NCW * 32;                 // consumer threads
constexpr int NTHREADS = NCT + 32;            // + producer warp
constexpr int STAGE_BYTES = MQ_STAGE_BYTES;   // ring stage (bulk copy) size
constexpr int NSTAGE = MQ_NSTAGE;             // ring depth
// Weight rows are placed in the ring at a stride of (row bytes + ROW_SKEW): the
// 16-byte skew puts consecutive rows in different shared-memory bank groups, so
// ldmatrix over 8 rows is conflict-free.  16 int8 rows of 1024 fill a stage.
constexpr int ROW_SKEW = 16;
constexpr int KV_CHUNK_POS = (STAGE_BYTES / (2 * HD * 2)) < 32 ? (STAGE_BYTES / (2 * HD * 2)) : 32;  // positions of K then V per chunk
constexpr int KV_V_OFFSET = KV_CHUNK_POS * HD * 2;  // V rows follow the K rows in a chunk
constexpr int MAX_SPLITS = 18;                // attention splits per KV head
constexpr int MAX_DEV_STATIC = 64;            // devices tracked by the allocation-free entry point
constexpr int MAX_LAYERS = 32;                // pointer/scale tables staged in shared memory
constexpr int MIN_CTAS = 148;                 // row shares below assume >= 148 CTAs (B200)
constexpr int QKV_MAXR = (QKV_ROWS + MIN_CTAS - 1) / MIN_CTAS;   // 28 rows per CTA
constexpr int O_MAXR = (HIDDEN + MIN_CTAS - 1) / MIN_CTAS;       // 7
constexpr int GU_MAXR = (INTER + MIN_CTAS - 1) / MIN_CTAS;       // 21
constexpr int LM_MAXR = (VOCAB + MIN_CTAS - 1) / MIN_CTAS;       // 1027
constexpr int SCL_O = QKV_MAXR, SCL_G = SCL_O + O_MAXR, SCL_U = SCL_G + GU_MAXR, SCL_D = SCL_U + GU_MAXR;
constexpr int SCL_STRIDE = SCL_D + O_MAXR;                       // 84 scales per layer per CTA

// ---------------------------------------------------------------------------
// Tagged hand-off words.  A value crossing CTAs is published as one 64-bit
// store (tag << 32 | payload).  An aligned 64-bit store is single-copy atomic,
// so a consumer that reads the expected tag also reads the matching payload;
// no fence or grid barrier is needed on the critical path.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_tagged(uint64_t* p, uint32_t tag, uint32_t payload) {
    uint64_t v = ((uint64_t)tag << 32) | payload;
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_relaxed32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Programmatic dependent launch: let the next grid on the stream be scheduled /
// wait until the previous grid has completed and its writes are visible.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------
// mbarrier + bulk copy (TMA engine, untiled, no multicast)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
// n arrivals at once (completes the phase of a barrier initialised with count n)
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.arrive.shared.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// 2-D tiled TMA load of one box at element coordinates (x, y) of the tensor map (x * element size must
// be a multiple of 16 bytes).
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void named_bar(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b16) { return __uint_as_float(b16 << 16); }
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float f) {
    return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Orderable key for a float: larger float -> larger unsigned key.
__device__ __forceinline__ uint32_t float_order_key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---------------------------------------------------------------------------
// Weight-type traits: how many elements a 16-byte unit holds and how to
// accumulate a unit against fp32 activations held in registers.
// ---------------------------------------------------------------------------
struct W8 {
    static constexpr int EPU = 16;  // int8 elements per 16-byte unit
    static constexpr bool HAS_SCALE = true;
    static constexpr bool LIMBS = true;   // matvecs use the Limbs dp4a path
    // int8 -> fp32 exactly: byte^0x80 placed in the mantissa of 2^23, minus 2^23+128.
    __device__ __forceinline__ static void dot(const uint4 w, const float* x, float& a0, float& a1) {
        const uint32_t ws[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u,
                                w.w ^ 0x80808080u};
#pragma unroll
        for (int j = 0; j < 4; j++) {
#pragma unroll
            for (int b = 0; b < 4; b++) {
                float f = __uint_as_float(__byte_perm(ws[j], 0x4B000000u, 0x7650 | b)) - 8388736.f;
                if (j & 1) a1 = fmaf(f, x[j * 4 + b], a1);
                else a0 = fmaf(f, x[j * 4 + b], a0);
            }
        }
    }
};
// Exact-integer INT8 dot product against fp32 activations.  Once per matvec
// phase the CTA scales the activation vector by one power of two 2^k (chosen
// so max|x| * 2^k < 2^22), rounds to integers X and splits each X into three
// signed 8-bit limbs, X = X2*2^16 + X1*2^8 + X0 (packed 4 per word, in shared
// memory).  A 16-byte weight unit then costs three dp4a per 4-byte word with
// exact int32 accumulation; each lane's partial sum is recombined exactly in
// fp64 and scaled back by 2^-k before the fp32 warp reduction.  The only
// rounding beyond fp32 summation is that of x to 22 bits relative to max|x|.
__device__ __forceinline__ void limb_split(float x, float up, uint32_t& p0, uint32_t& p1, uint32_t& p2, int b) {
    const int X = __float2int_rn(x * up);
    const int d0 = ((X + 128) & 255) - 128;
    const int r = (X - d0) >> 8;
    const int d1 = ((r + 128) & 255) - 128;
    const int d2 = (r - d1) >> 8;
    p0 |= (uint32_t)(d0 & 255) << (8 * b);
    p1 |= (uint32_t)(d1 & 255) << (8 * b);
    p2 |= (uint32_t)(d2 & 255) << (8 * b);
}
// Power-of-two scale for max|x| = m: returns 2^k, sets inv = 2^-k.
__device__ __forceinline__ float limb_scale(float m, float& inv) {
    int e = 0;
    frexpf(m, &e);                      // m < 2^e
    int k = m > 0.f ? 22 - e : 0;
    k = max(-126, min(126, k));
    inv = __int_as_float((127 - k) << 23);
    return __int_as_float((127 + k) << 23);
}
template <int NW>   // NW = 4-byte activation words per lane (K / 128)
struct Limbs {
    int l0[NW], l1[NW], l2[NW];
    float inv;  // 2^-k
    // Loads this lane's words: unit j of the lane covers words 4*(lane+32j) .. +3.
    __device__ __forceinline__ void load(const int* L0, const int* L1, const int* L2, int lane, float inv_) {
        inv = inv_;
#pragma unroll
        for (int j = 0; j < NW / 4; ++j) {
            const int w = 4 * (lane + 32 * j);
            const int4 a = *reinterpret_cast<const int4*>(L0 + w);
            const int4 b = *reinterpret_cast<const int4*>(L1 + w);
            const int4 c = *reinterpret_cast<const int4*>(L2 + w);
            l0[4 * j] = a.x; l0[4 * j + 1] = a.y; l0[4 * j + 2] = a.z; l0[4 * j + 3] = a.w;
            l1[4 * j] = b.x; l1[4 * j + 1] = b.y; l1[4 * j + 2] = b.z; l1[4 * j + 3] = b.w;
            l2[4 * j] = c.x; l2[4 * j + 1] = c.y; l2[4 * j + 2] = c.z; l2[4 * j + 3] = c.w;
        }
    }
    // Dot of this lane's limbs with the int8 weights of unit j (words 4j..4j+3).
    __device__ __forceinline__ void acc(const uint4 w, int j, int& a0, int& a1, int& a2) const {
        a0 = __dp4a((int)w.x, l0[4 * j + 0], a0); a1 = __dp4a((int)w.x, l1[4 * j + 0], a1); a2 = __dp4a((int)w.x, l2[4 * j + 0], a2);
        a0 = __dp4a((int)w.y, l0[4 * j + 1], a0); a1 = __dp4a((int)w.y, l1[4 * j + 1], a1); a2 = __dp4a((int)w.y, l2[4 * j + 1], a2);
        a0 = __dp4a((int)w.z, l0[4 * j + 2], a0); a1 = __dp4a((int)w.z, l1[4 * j + 2], a1); a2 = __dp4a((int)w.z, l2[4 * j + 2], a2);
        a0 = __dp4a((int)w.w, l0[4 * j + 3], a0); a1 = __dp4a((int)w.w, l1[4 * j + 3], a1); a2 = __dp4a((int)w.w, l2[4 * j + 3], a2);
    }
    __device__ __forceinline__ float finish(int a0, int a1, int a2) const {
        const double v = fma((double)a2, 65536.0, fma((double)a1, 256.0, (double)a0));  // exact (< 2^53)
        return (float)v * inv;
    }
};

struct W16 {
    static constexpr int EPU = 8;  // bf16 elements per 16-byte unit
    static constexpr bool HAS_SCALE = false;
    static constexpr bool LIMBS = false;
    __device__ __forceinline__ static void dot(const uint4 w, const float* x, float& a0, float& a1) {
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float lo = __uint_as_float(ws[j] << 16);
            float hi = __uint_as_float(ws[j] & 0xffff0000u);
            if (j & 1) { a1 = fmaf(lo, x[2 * j], a1); a1 = fmaf(hi, x[2 * j + 1], a1); }
            else       { a0 = fmaf(lo, x[2 * j], a0); a0 = fmaf(hi, x[2 * j + 1], a0); }
        }
    }
};

__host__ __device__ __forceinline__ int split_lo(int n, int parts, int i) {
    return (int)(((long long)n * i) / parts);
}

}  // namespace mq
