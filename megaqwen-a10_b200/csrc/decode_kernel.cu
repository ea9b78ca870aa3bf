// decode_kernel.cu -- persistent fused Qwen3-0.6B decode step for B200 (sm_100a).
//
// One launch = one greedy decode step: embedding -> num_layers x {RMSNorm+QKV,
// QK-norm+RoPE+KV write, attention, O+residual, post-norm+gate/up+SiLU,
// down+residual} -> final RMSNorm -> LM head + argmax.  This is the computation
// of the reference's a10_decode_kernel + lm_head_phase1/2
// (a10_int8_decode_kernel.cu:621-815) re-designed for B200:
//   * one CTA per SM (148), NCW consumer warps + 1 producer warp;
//   * the producer streams this CTA's weight rows (and KV rows for its attention
//     split) through an NSTAGE x 16 KB shared-memory ring with cp.async.bulk, so
//     HBM reads run ahead of the data dependencies;
//   * no grid.sync: each cross-CTA value is a tagged 64-bit word and a consumer
//     polls exactly the words it needs (see common.cuh);
//   * every norm is recomputed per CTA instead of by CTA 0 plus a barrier;
//   * attention is split over positions (flash-decode) with an online softmax,
//     one work item per (KV head, split), both GQA heads of a KV head at once;
//   * the LM head runs inside the same launch and reduces its argmax with one
//     packed 64-bit atomicMax per CTA.
// Every spin is bounded by a %globaltimer budget; on expiry the kernel records
// an MQ_DEV_* code in the workspace, drains its bulk copies and returns.
#include "decode.cuh"
#include <stdlib.h>

// MQ_PHASE_NOINLINE=1 keeps the phase bodies out of line (smaller kernel code).
#if defined(MQ_PHASE_NOINLINE) && MQ_PHASE_NOINLINE
#define MQ_PHASE __device__ __noinline__
#else
#define MQ_PHASE __device__ __forceinline__
#endif


namespace mq {

struct Ctx {
    Smem* sm;
    Workspace* ws;
    unsigned long long budget;
};

__device__ __noinline__ void record_error(Ctx& c, int code, int info) {
    if (atomicCAS(&c.ws->err_code, 0, code) == 0) atomicExch(&c.ws->err_info, info);
    *(volatile int*)&c.sm->abort_flag = 1;
}

__device__ __forceinline__ bool aborted(Ctx& c) {
    if (*(volatile int*)&c.sm->abort_flag) return true;
    if (ld_relaxed32((const uint32_t*)&c.ws->err_code) != 0) {
        *(volatile int*)&c.sm->abort_flag = 1;
        return true;
    }
    return false;
}

// Poll one tagged word until its tag matches.  Returns the payload; on abort or
// timeout returns 0 (the caller's CTA then leaves at the next phase boundary).
__device__ __forceinline__ uint32_t poll_word(Ctx& c, const uint64_t* p, uint32_t tag, int where) {
    uint64_t v = ld_relaxed64(p);
    if ((uint32_t)(v >> 32) == tag) return (uint32_t)v;
    unsigned long long t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        v = ld_relaxed64(p);
        if ((uint32_t)(v >> 32) == tag) return (uint32_t)v;
        if ((it & 127) == 0) {
            if (aborted(c)) return 0;
            if (globaltimer() - t0 > c.budget) {
                record_error(c, MQ_DEV_TIMEOUT_EXCHANGE, where);
                return 0;
            }
        }
    }
}

// `budget_mul` lets the producer wait longer than the consumers: a producer
// stalled on a full ring is a consequence of a stalled consumer, whose own
// timeout is the root cause worth recording.
__device__ __forceinline__ bool mbar_wait(Ctx& c, uint64_t* b, uint32_t parity, int where, int budget_mul = 1) {
    if (mbar_test(b, parity)) return true;
    unsigned long long t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_test(b, parity)) return true;
        if ((it & 63) == 0) {
            if (aborted(c)) return false;
            if (globaltimer() - t0 > c.budget * budget_mul) {
                record_error(c, MQ_DEV_TIMEOUT_RING, where);
                return false;
            }
        }
    }
}

// Consumer-side barrier with an OR-reduction: every consumer thread gets the same
// answer to "has any thread seen an abort".
__device__ __forceinline__ bool consumers_sync_abort(Ctx& c) {
    int mine = *(volatile int*)&c.sm->abort_flag;
    int any;
    asm volatile(
        "{ .reg .pred p, q; setp.ne.s32 p, %1, 0; bar.red.or.pred q, 1, %2, p; selp.s32 %0, 1, 0, q; }"
        : "=r"(any)
        : "r"(mine), "r"(NCT)
        : "memory");
    return any != 0;
}
__device__ __forceinline__ void consumers_sync() { named_bar(1, NCT); }

// ---------------------------------------------------------------------------
// Work geometry, shared by producer and consumers so both walk the same chunks.
// ---------------------------------------------------------------------------
struct Geo {
    int nb, b;
    int qkv0, qkv1, o0, o1, gu0, gu1, d0, d1, lm0, lm1;
    int item, g, s, S;
    int c;                  // cache_len
    int past0, past1;       // cache positions this split reads from the cache
    bool owner;             // split that holds the current position

    __device__ void init(const DecodeParams& P) {
        nb = gridDim.x;
        b = blockIdx.x;
        qkv0 = split_lo(QKV_ROWS, nb, b); qkv1 = split_lo(QKV_ROWS, nb, b + 1);
        o0 = split_lo(HIDDEN, nb, b);     o1 = split_lo(HIDDEN, nb, b + 1);
        gu0 = split_lo(INTER, nb, b);     gu1 = split_lo(INTER, nb, b + 1);
        d0 = o0; d1 = o1;
        lm0 = split_lo(VOCAB, nb, b);     lm1 = split_lo(VOCAB, nb, b + 1);
        S = P.splits;
        c = P.position + 1;
        const int nitems = NKVH * S;
        const int stride = nb / nitems;
        item = (b % stride == 0 && b / stride < nitems) ? b / stride : -1;
        if (item >= 0) {
            g = item / S;
            s = item % S;
            int p0 = split_lo(c, S, s), p1 = split_lo(c, S, s + 1);
            owner = (s == S - 1);
            past0 = p0;
            past1 = owner ? c - 1 : p1;
        } else {
            g = s = 0; owner = false; past0 = past1 = 0;
        }
    }
};

template <class WT>
struct Bytes {
    static constexpr int ESZ = 16 / WT::EPU;  // bytes per weight element
};

// ---------------------------------------------------------------------------
// Producer: one thread walks the CTA's chunk sequence for the whole step.
// ---------------------------------------------------------------------------
struct Producer {
    Smem* sm;
    uint32_t seq;
    int pad;  // global row padding: 0 (dense rows, one copy per row) or ROW_SKEW (one copy per run)

    // Copies rows [a, b) of a matrix with rb payload bytes per row into dst at a
    // stride of rb + ROW_SKEW.  With padded rows the global layout already has
    // that stride and the run is one bulk copy.
    __device__ void run(uint8_t* dst, const uint8_t* base, int a, int n, int rb, uint64_t* bar) {
        const int rs = rb + ROW_SKEW;
        if (pad) {
            bulk_g2s(dst, base + (size_t)a * rs, n * rs, bar);
        } else {
            for (int i = 0; i < n; ++i) bulk_g2s(dst + i * rs, base + (size_t)(a + i) * rb, rb, bar);
        }
    }
    __device__ uint32_t bytes(int n, int rb) const { return pad ? n * (rb + ROW_SKEW) : n * rb; }

    __device__ bool begin(Ctx& c, uint32_t bytes, uint8_t*& dst) {
        const uint32_t stage = seq % NSTAGE, use = seq / NSTAGE;
        if (use > 0 && !mbar_wait(c, &sm->empty[stage], (use - 1) & 1, 100 + (int)stage, 2)) return false;
        mbar_arrive_expect_tx(&sm->full[stage], bytes);
        dst = sm->ring[stage];
        return true;
    }
    __device__ void end() { ++seq; }

    // rows [a, b) of a row-major matrix with `rb` bytes per row, placed in the
    // stage at a stride of rb + ROW_SKEW (one bulk copy per row).
    __device__ bool rows(Ctx& c, const uint8_t* base, int a, int b, int rb) {
        const int rs = rb + ROW_SKEW, rpc = STAGE_BYTES / rs;
        for (int r = a; r < b; r += rpc) {
            const int n = min(rpc, b - r);
            uint8_t* dst;
            if (!begin(c, bytes(n, rb), dst)) return false;
            run(dst, base, r, n, rb, &sm->full[seq % NSTAGE]);
            end();
        }
        return true;
    }
};

template <class WT>
__device__ void producer_main(const DecodeParams& P, Ctx& c, const Geo& G) {
    constexpr int ESZ = Bytes<WT>::ESZ;
    Producer pr{c.sm, 0, P.row_pad};
    bool ok = true;
    // L2 prefetch of the first kv_pf_pos cached positions of layer l's split,
    // issued one layer ahead: the copies run while the HBM is otherwise lightly
    // used (the matvec phases), and the layer's ring copies then hit L2.
    auto prefetch_kv = [&](int l) {
        if (G.item < 0 || P.kv_pf_pos <= 0 || l >= P.L) return;
        const int n = min(P.kv_pf_pos, G.past1 - G.past0);
        const size_t off = (((size_t)l * NKVH + G.g) * (size_t)P.max_seq + G.past0) * HD;
        for (int p = 0; p < n; p += 128) {
            const uint32_t bytes = (uint32_t)min(128, n - p) * HD * 2;
            prefetch_l2(P.kc + off + (size_t)p * HD, bytes);
            prefetch_l2(P.vc + off + (size_t)p * HD, bytes);
        }
    };
    prefetch_kv(0);
    for (int l = 0; l < P.L && ok; ++l) {
        const LayerWeights& w = P.layers[l];
        // QKV rows in the stacked [q; k; v] row space.
        {
            const int rb = HIDDEN * ESZ, rs = rb + ROW_SKEW, rpc = STAGE_BYTES / rs;
            for (int r = G.qkv0; r < G.qkv1 && ok; r += rpc) {
                const int n = min(rpc, G.qkv1 - r);
                uint8_t* dst;
                if (!(ok = pr.begin(c, pr.bytes(n, rb), dst))) break;
                uint64_t* bar = &c.sm->full[pr.seq % NSTAGE];
                int done = 0;
                while (done < n) {  // runs within the q, k and v matrices
                    const int row = r + done;
                    const uint8_t* base;
                    int first, lim;
                    if (row < QSZ) { base = (const uint8_t*)w.q_proj_weight; first = 0; lim = QSZ; }
                    else if (row < QSZ + KVSZ) { base = (const uint8_t*)w.k_proj_weight; first = QSZ; lim = QSZ + KVSZ; }
                    else { base = (const uint8_t*)w.v_proj_weight; first = QSZ + KVSZ; lim = QKV_ROWS; }
                    const int m = min(n - done, lim - row);
                    pr.run(dst + done * rs, base, row - first, m, rb, bar);
                    done += m;
                }
                pr.end();
            }
        }
        // KV rows of this CTA's attention split (positions written by earlier launches).
        if (ok && G.item >= 0) {
            if (l == 0) pdl_wait();   // cache rows written by the previous step
            const size_t head_off = ((size_t)l * NKVH + G.g) * (size_t)P.max_seq * HD;
            for (int p = G.past0; p < G.past1 && ok; p += KV_CHUNK_POS) {
                const int n = min(KV_CHUNK_POS, G.past1 - p);
                uint8_t* dst;
                if (!(ok = pr.begin(c, 2 * n * HD * 2, dst))) break;
                uint64_t* bar = &c.sm->full[pr.seq % NSTAGE];
                bulk_g2s(dst, P.kc + head_off + (size_t)p * HD, n * HD * 2, bar);
                bulk_g2s(dst + KV_V_OFFSET, P.vc + head_off + (size_t)p * HD, n * HD * 2, bar);
                pr.end();
            }
            prefetch_kv(l + 1);
        }
        if (ok) ok = pr.rows(c, (const uint8_t*)w.o_proj_weight, G.o0, G.o1, QSZ * ESZ);
        // gate/up: a chunk holds n gate rows followed by the same n up rows.
        if (ok) {
            const int rb = HIDDEN * ESZ, rs = rb + ROW_SKEW, rpc = STAGE_BYTES / (2 * rs);
            for (int r = G.gu0; r < G.gu1 && ok; r += rpc) {
                const int n = min(rpc, G.gu1 - r);
                uint8_t* dst;
                if (!(ok = pr.begin(c, 2 * pr.bytes(n, rb), dst))) break;
                uint64_t* bar = &c.sm->full[pr.seq % NSTAGE];
                pr.run(dst, (const uint8_t*)w.gate_proj_weight, r, n, rb, bar);
                pr.run(dst + n * rs, (const uint8_t*)w.up_proj_weight, r, n, rb, bar);
                pr.end();
            }
        }
        if (ok) ok = pr.rows(c, (const uint8_t*)w.down_proj_weight, G.d0, G.d1, INTER * ESZ);
    }
    if (ok) pr.rows(c, (const uint8_t*)P.lm_w, G.lm0, G.lm1, HIDDEN * ESZ);
    // Drain: never leave a bulk copy in flight into shared memory at exit.
    const uint32_t first = pr.seq > (uint32_t)NSTAGE ? pr.seq - NSTAGE : 0u;
    for (uint32_t q = first; q < pr.seq; ++q) {
        const uint32_t stage = q % NSTAGE;
        unsigned long long t0 = globaltimer();
        while (!mbar_test(&c.sm->full[stage], (q / NSTAGE) & 1)) {
            if (globaltimer() - t0 > c.budget) break;
        }
    }
}


// ---------------------------------------------------------------------------
// Consumer side
// ---------------------------------------------------------------------------
struct Cons {
    Smem* sm;
    uint32_t seq;
    int warp, lane, tid;


    __device__ const uint8_t* wait(Ctx& c, int where) {
        const uint32_t stage = seq % NSTAGE;
        mbar_wait(c, &sm->full[stage], (seq / NSTAGE) & 1, where);
        return sm->ring[stage];
    }
    __device__ void release() {
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm->empty[seq % NSTAGE]);
        ++seq;
    }
    // A chunk that only this warp reads: its arrival stands for all NCW warps, and
    // the other warps step past it with skip(), so the stage is free as soon as
    // its one reader is done with it.
    // Used only where every chunk of a stage has the same single reader: a reader that
    // skipped ahead could otherwise test a stage's parity a whole ring early.
    __device__ void release_owned() {
        __syncwarp();
        if (lane == 0) mbar_arrive_cnt(&sm->empty[seq % NSTAGE], NCW);
        ++seq;
    }
    __device__ void skip() { ++seq; }
    // The q-th chunk after the next one (q = 0 is what wait() would return).
    __device__ const uint8_t* wait_at(Ctx& c, uint32_t q, int where) {
        const uint32_t s = seq + q, stage = s % NSTAGE;
        mbar_wait(c, &sm->full[stage], (s / NSTAGE) & 1, where);
        return sm->ring[stage];
    }
    // Releases the next n chunks (after wait_at on each of them).
    __device__ void release_n(uint32_t n) {
        __syncwarp();
        if (lane == 0)
            for (uint32_t q = 0; q < n; ++q) mbar_arrive(&sm->empty[(seq + q) % NSTAGE]);
        seq += n;
    }
};

// Matvec over rows [r0, r1) of one projection streamed through the ring.
// Row i (phase-relative) is handled by warp i % NCW; lane holds the activation
// elements of its fixed 16-byte units in registers for the whole phase.
// Builds the limbs of x_s[0..n) into shared memory (all consumer threads; the
// caller guarantees x_s is complete).  Two consumer barriers.
MQ_PHASE void build_limbs(Cons& cs, const float* x_s, int n) {
    Smem* sm = cs.sm;
    float m = 0.f;
    for (int i = cs.tid; i < n; i += NCT) m = fmaxf(m, fabsf(x_s[i]));
    m = warp_max(m);
    if (cs.lane == 0) sm->red2[cs.warp] = m;
    consumers_sync();
#pragma unroll
    for (int i = 0; i < NCW; ++i) m = fmaxf(m, sm->red2[i]);
    float inv;
    const float up = limb_scale(m, inv);
    for (int w = cs.tid; w < n / 4; w += NCT) {
        const float4 v = *reinterpret_cast<const float4*>(x_s + 4 * w);
        uint32_t p0 = 0, p1 = 0, p2 = 0;
        limb_split(v.x, up, p0, p1, p2, 0);
        limb_split(v.y, up, p0, p1, p2, 1);
        limb_split(v.z, up, p0, p1, p2, 2);
        limb_split(v.w, up, p0, p1, p2, 3);
        sm->limb[0][w] = (int)p0; sm->limb[1][w] = (int)p1; sm->limb[2][w] = (int)p2; sm->limb[3][w] = 0;
    }
    if (cs.tid == 0) sm->limb_inv = inv;
    consumers_sync();
}

template <class WT, int K, class Scl, class Out>
MQ_PHASE void mv_phase(Ctx& c, Cons& cs, int r0, int r1, const float* x_s, Scl scl, Out out) {
    constexpr int ESZ = Bytes<WT>::ESZ;
    constexpr int RB = K * ESZ;
    constexpr int UPL = K / (WT::EPU * 32);
    constexpr int RS = RB + ROW_SKEW;
    constexpr int RPC = STAGE_BYTES / RS;
    float xr[WT::LIMBS ? 1 : UPL * WT::EPU];
    Limbs<WT::LIMBS ? UPL * 4 : 4> lb;
    if constexpr (WT::LIMBS) {
        build_limbs(cs, x_s, K);
        lb.load(cs.sm->limb[0], cs.sm->limb[1], cs.sm->limb[2], cs.lane, cs.sm->limb_inv);
    } else {
#pragma unroll
        for (int j = 0; j < UPL; ++j) {
            const int e0 = (cs.lane + 32 * j) * WT::EPU;
#pragma unroll
            for (int e = 0; e < WT::EPU; e += 4) {
                float4 v = *reinterpret_cast<const float4*>(x_s + e0 + e);
                xr[j * WT::EPU + e] = v.x; xr[j * WT::EPU + e + 1] = v.y;
                xr[j * WT::EPU + e + 2] = v.z; xr[j * WT::EPU + e + 3] = v.w;
            }
        }
    }
    const int n = r1 - r0;
    for (int cb = 0; cb < n; cb += RPC) {
        const int ce = min(n, cb + RPC);
        const uint8_t* st = cs.wait(c, 1);
        int i = cb + ((cs.warp - cb) % NCW + NCW) % NCW;
        for (; i < ce; i += NCW) {
            const float sc = scl(r0 + i);
            const uint4* row = reinterpret_cast<const uint4*>(st + (size_t)(i - cb) * RS);
            float part;
            if constexpr (WT::LIMBS) {
                int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
                for (int j = 0; j < UPL; ++j) lb.acc(row[cs.lane + 32 * j], j, a0, a1, a2);
                part = lb.finish(a0, a1, a2);
            } else {
                float a0 = 0.f, a1 = 0.f;
#pragma unroll
                for (int j = 0; j < UPL; ++j) WT::dot(row[cs.lane + 32 * j], xr + j * WT::EPU, a0, a1);
                part = a0 + a1;
            }
            const float dot = warp_sum(part);
            if (cs.lane == 0) out(r0 + i, dot * sc);
        }
        cs.release();
    }
}

// gate/up pair phase: out(i, gate_dot, up_dot).
template <class WT, class Out>
MQ_PHASE void gu_phase(Ctx& c, Cons& cs, int r0, int r1, const float* x_s, const float* sg,
                                         const float* su, Out out) {
    constexpr int K = HIDDEN;
    constexpr int ESZ = Bytes<WT>::ESZ;
    constexpr int RB = K * ESZ;
    constexpr int UPL = K / (WT::EPU * 32);
    constexpr int RS = RB + ROW_SKEW;
    constexpr int RPC = STAGE_BYTES / (2 * RS);
    float xr[WT::LIMBS ? 1 : UPL * WT::EPU];
    Limbs<WT::LIMBS ? UPL * 4 : 4> lb;
    if constexpr (WT::LIMBS) {
        build_limbs(cs, x_s, K);
        lb.load(cs.sm->limb[0], cs.sm->limb[1], cs.sm->limb[2], cs.lane, cs.sm->limb_inv);
    } else {
#pragma unroll
        for (int j = 0; j < UPL; ++j) {
            const int e0 = (cs.lane + 32 * j) * WT::EPU;
#pragma unroll
            for (int e = 0; e < WT::EPU; e += 4) {
                float4 v = *reinterpret_cast<const float4*>(x_s + e0 + e);
                xr[j * WT::EPU + e] = v.x; xr[j * WT::EPU + e + 1] = v.y;
                xr[j * WT::EPU + e + 2] = v.z; xr[j * WT::EPU + e + 3] = v.w;
            }
        }
    }
    const int n = r1 - r0;
    for (int cb = 0; cb < n; cb += RPC) {
        const int ce = min(n, cb + RPC);
        const int nin = ce - cb;
        const uint8_t* st = cs.wait(c, 2);
        int i = cb + ((cs.warp - cb) % NCW + NCW) % NCW;
        for (; i < ce; i += NCW) {
            float gsc = 1.f, usc = 1.f;
            if (WT::HAS_SCALE) { gsc = sg[i]; usc = su[i]; }  // phase-relative, shared memory
            const uint4* grow = reinterpret_cast<const uint4*>(st + (size_t)(i - cb) * RS);
            const uint4* urow = reinterpret_cast<const uint4*>(st + (size_t)(nin + i - cb) * RS);
            float gp, up;
            if constexpr (WT::LIMBS) {
                int g0 = 0, g1 = 0, g2 = 0, u0 = 0, u1 = 0, u2 = 0;
#pragma unroll
                for (int j = 0; j < UPL; ++j) {
                    lb.acc(grow[cs.lane + 32 * j], j, g0, g1, g2);
                    lb.acc(urow[cs.lane + 32 * j], j, u0, u1, u2);
                }
                gp = lb.finish(g0, g1, g2);
                up = lb.finish(u0, u1, u2);
            } else {
                float g0 = 0.f, g1 = 0.f, u0 = 0.f, u1 = 0.f;
#pragma unroll
                for (int j = 0; j < UPL; ++j) {
                    WT::dot(grow[cs.lane + 32 * j], xr + j * WT::EPU, g0, g1);
                    WT::dot(urow[cs.lane + 32 * j], xr + j * WT::EPU, u0, u1);
                }
                gp = g0 + g1;
                up = u0 + u1;
            }
            const float gd = warp_sum(gp);
            const float ud = warp_sum(up);
            if (cs.lane == 0) out(r0 + i, gd * gsc, ud * usc);
        }
        cs.release();
    }
}

// ---------------------------------------------------------------------------
// INT8 matvec on the tensor cores for the throughput-bound LM head (and the
// stand-alone mq_matvec), exact: mma.sync m16n8k32 s8 x s8 -> s32 with
// A = 16 weight rows x 32 bytes (ldmatrix from the skewed ring rows) and
// B = the activation limbs (column n of B = limb n for n < 3, zero otherwise).
// The int32 results are the same exact integers the dp4a formulation yields.
// The latency-bound per-layer phases use the dp4a path (mv_phase / gu_phase):
// a dependent mma.sync chain of a few steps is slower there.
// ---------------------------------------------------------------------------
// st[q] for a runtime q without dynamic register-array indexing.
template <int N>
__device__ __forceinline__ const uint8_t* pick(const uint8_t* const (&st)[N], int q) {
    const uint8_t* r = st[0];
#pragma unroll
    for (int k = 1; k < N; ++k) r = (q == k) ? st[k] : r;
    return r;
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// This lane's ldmatrix row address for tile row tr (lanes 0-7: rows 0-7 bytes
// 0-15, 8-15: rows 8-15 bytes 0-15, 16-23: rows 0-7 bytes 16-31, 24-31: rows 8-15).
__device__ __forceinline__ int mma_lane_row(int lane) { return (lane & 7) + 8 * ((lane >> 3) & 1); }
__device__ __forceinline__ int mma_lane_koff(int lane) { return 16 * (lane >> 4); }

__device__ __forceinline__ float limb_finish(long long a0, long long a1, long long a2, float inv) {
    const double v = fma((double)a2, 65536.0, fma((double)a1, 256.0, (double)a0));
    return (float)v * inv;
}

// Streaming phase (LM head, stand-alone matvec): every ring chunk is one tile
// (<= 16 rows) done by one warp (chunk q -> warp q % NCW) over all k-steps.
// out(row, value) is called by lanes t == 0 (two rows each).
// The limbs of the activation (scale 2^-k = inv) are already in shared memory
// (sm->limb rows 0-2; row 3 all zero).
template <int K, class Scl, class Out>
__device__ __forceinline__ void mma_stream(Ctx& c, Cons& cs, int r0, int r1, float inv, Scl scl, Out out) {
    constexpr int RS = K + ROW_SKEW;
    constexpr int RPC = STAGE_BYTES / RS;
    constexpr int KS = K / 32;
    static_assert(RPC <= 16, "one tile per chunk");
    const int g = cs.lane >> 2, t = cs.lane & 3;
    const int* lb = cs.sm->limb[g < 3 ? g : 3];
    const int n = r1 - r0;
    for (int cb = 0, q = 0; cb < n; cb += RPC, ++q) {
        const uint8_t* st = cs.wait(c, 1);
        if (q % NCW == cs.warp) {
            const int rows = min(RPC, n - cb);
            const int tr = min(mma_lane_row(cs.lane), rows - 1);
            const uint32_t abase = smem_u32(st + (size_t)tr * RS) + mma_lane_koff(cs.lane);
            int d0[4] = {0, 0, 0, 0}, d1[4] = {0, 0, 0, 0};
#pragma unroll 4
            for (int ks = 0; ks < KS; ks += 2) {
                uint32_t a[4], b[4];
                ldmatrix_x4(a, abase + ks * 32);
                ldmatrix_x4(b, abase + ks * 32 + 32);
                mma_s8(d0, a, (uint32_t)lb[8 * ks + t], (uint32_t)lb[8 * ks + 4 + t]);
                mma_s8(d1, b, (uint32_t)lb[8 * ks + 8 + t], (uint32_t)lb[8 * ks + 12 + t]);
            }
            // limb 2 of rows g, g+8 lives in lane t == 1 (column 2)
            const int x0 = d0[0] + d1[0], x1 = d0[1] + d1[1], x2 = d0[2] + d1[2], x3 = d0[3] + d1[3];
            const int l2a = __shfl_down_sync(0xffffffffu, x0, 1);
            const int l2b = __shfl_down_sync(0xffffffffu, x2, 1);
            if (t == 0) {
                if (g < rows) out(r0 + cb + g, limb_finish(x0, x1, l2a, inv) * scl(r0 + cb + g));
                if (g + 8 < rows) out(r0 + cb + g + 8, limb_finish(x2, x3, l2b, inv) * scl(r0 + cb + g + 8));
            }
        }
        cs.release();
    }
}



// ---------------------------------------------------------------------------
// Exchange gather that leaves the next matvec's input ready.
//
// Thread t owns the groups of four consecutive words g = t, t + NCT, ... of an
// n-word exchange.  It polls them with one 32-byte load per group and round
// (the number of poll requests, not their size, sets the exchange latency:
// 8-byte polls cost ~13 us per layer more than 32-byte ones), and forms v_i (the
// payload as fp32) and y_i = v_i * w_i (w: the RMSNorm weight of the next
// matvec, or 1).  y goes to xs (fp32, shared memory), v to keep when given.  One
// consumer barrier reduces, in a fixed order, max|y| (the limb scale 2^k) and,
// for a normalised input, sum(v^2) (rstd = rsqrt(mean + eps)); then every
// thread splits its own y values into the three int8 limbs of y * 2^k and a
// second barrier publishes them.  The norm's rstd is applied to the matvec
// outputs: W (v * w * rstd) = rstd * W (v * w).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ld_relaxed_v4(const uint64_t* p, uint64_t (&v)[4]) {
    asm volatile("ld.relaxed.gpu.global.v4.b64 {%0, %1, %2, %3}, [%4];"
                 : "=l"(v[0]), "=l"(v[1]), "=l"(v[2]), "=l"(v[3]) : "l"(p) : "memory");
}

// Each 8-byte word of the vector access is single-copy atomic, so a word's tag
// and payload arrive together.
template <int MAXG, class Addr>
__device__ __forceinline__ void poll_groups_at(Ctx& c, const Cons& cs, Addr addr, int ngroups, uint32_t tag,
                                               int where, uint32_t (&pay)[MAXG][4]) {
    uint64_t v[MAXG][4];
#pragma unroll
    for (int k = 0; k < MAXG; ++k) {
        const int g = cs.tid + k * NCT;
        if (g < ngroups) ld_relaxed_v4(addr(g), v[k]);
        else v[k][0] = v[k][1] = v[k][2] = v[k][3] = (uint64_t)tag << 32;
    }
    unsigned long long t0 = 0;
    for (uint32_t it = 0;; ++it) {
        bool done = true;
#pragma unroll
        for (int k = 0; k < MAXG; ++k) {
            const int g = cs.tid + k * NCT;
            if ((uint32_t)(v[k][0] >> 32) != tag || (uint32_t)(v[k][1] >> 32) != tag ||
                (uint32_t)(v[k][2] >> 32) != tag || (uint32_t)(v[k][3] >> 32) != tag) {
                done = false;
                ld_relaxed_v4(addr(g), v[k]);
            }
        }
        if (done) break;
        if ((it & 127) == 127) {
            if (t0 == 0) t0 = globaltimer();
            if (aborted(c)) break;
            if (globaltimer() - t0 > c.budget) { record_error(c, MQ_DEV_TIMEOUT_EXCHANGE, where); break; }
        }
    }
#pragma unroll
    for (int k = 0; k < MAXG; ++k)
#pragma unroll
        for (int e = 0; e < 4; ++e) pay[k][e] = (uint32_t)v[k][e];
}

// addr(g): the 4 consecutive words of group g.
template <int MAXG>
__device__ __forceinline__ void poll_groups(Ctx& c, const Cons& cs, const uint64_t* base, int ngroups, uint32_t tag,
                                            int where, uint32_t (&pay)[MAXG][4]) {
    poll_groups_at<MAXG>(c, cs, [&](int g) { return base + 4 * g; }, ngroups, tag, where, pay);
}

struct InputScale {
    float inv;   // 2^-k of the limbs (1 without limbs)
    float rstd;  // RMSNorm factor of a normalised input (1 otherwise)
};

// Norm weights of this thread's group (elements 4t .. 4t+3 of a 1024-wide
// vector), loaded one phase ahead of use and kept as raw bf16 pairs: converting
// at load time would make the thread wait for the load right there.
struct NormW4 {
    uint32_t raw[2];
    __device__ __forceinline__ void load(const Cons& cs, const void* w) {
        raw[0] = raw[1] = 0u;
        if (cs.tid < HIDDEN / 4) {
            const uint16_t* p = reinterpret_cast<const uint16_t*>(w) + 4 * cs.tid;
            if ((reinterpret_cast<uintptr_t>(p) & 7) == 0) {
                const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
                raw[0] = u.x; raw[1] = u.y;
            } else {
                raw[0] = (uint32_t)__ldg(p) | ((uint32_t)__ldg(p + 1) << 16);
                raw[1] = (uint32_t)__ldg(p + 2) | ((uint32_t)__ldg(p + 3) << 16);
            }
        }
    }
    __device__ __forceinline__ float get(int e) const {
        const uint32_t w = raw[e >> 1];
        return bf16_bits_to_f32((e & 1) ? (w >> 16) : (w & 0xffffu));
    }
};

// Second half of the gather: payloads (bf16 bits or fp32 bits) -> xs / keep /
// limbs as described above.  NORM requires ngroups == HIDDEN / 4 (MAXG == 1).
// LIMBS: two consumer barriers; otherwise one.
template <int MAXG, bool LIMBS, bool NORM>
MQ_PHASE InputScale finish_input(Cons& cs, const uint32_t (&pay)[MAXG][4], int ngroups, bool bf16pay,
                                 const NormW4& w, float* xs, float* keep) {
    static_assert(!NORM || MAXG == 1, "normalised inputs are 1024 wide");
    Smem* sm = cs.sm;
    float y[MAXG][4];
    float mx = 0.f, ss = 0.f;
#pragma unroll
    for (int k = 0; k < MAXG; ++k) {
        const int g = cs.tid + k * NCT;
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            v[e] = bf16pay ? bf16_bits_to_f32(pay[k][e] & 0xffffu) : __uint_as_float(pay[k][e]);
            if (g >= ngroups) v[e] = 0.f;
            ss = fmaf(v[e], v[e], ss);
            y[k][e] = NORM ? v[e] * w.get(e) : v[e];
            mx = fmaxf(mx, fabsf(y[k][e]));
        }
        if (g < ngroups) {
            *reinterpret_cast<float4*>(xs + 4 * g) = make_float4(y[k][0], y[k][1], y[k][2], y[k][3]);
            if (keep) *reinterpret_cast<float4*>(keep + 4 * g) = make_float4(v[0], v[1], v[2], v[3]);
        }
    }
    if (LIMBS) mx = warp_max(mx);
    if (NORM) ss = warp_sum(ss);
    if (cs.lane == 0) { sm->red[cs.warp] = ss; sm->red2[cs.warp] = mx; }
    consumers_sync();
    InputScale out{1.f, 1.f};
    if (NORM) {
        float tot = 0.f;
#pragma unroll
        for (int i = 0; i < NCW; ++i) tot += sm->red[i];
        out.rstd = rsqrtf(tot / (float)HIDDEN + RMS_EPS);
    }
    if (LIMBS) {
        float m = 0.f;
#pragma unroll
        for (int i = 0; i < NCW; ++i) m = fmaxf(m, sm->red2[i]);
        float inv;
        const float up = limb_scale(m, inv);
        out.inv = inv;
#pragma unroll
        for (int k = 0; k < MAXG; ++k) {
            const int g = cs.tid + k * NCT;
            if (g < ngroups) {
                uint32_t p0 = 0, p1 = 0, p2 = 0;
#pragma unroll
                for (int e = 0; e < 4; ++e) limb_split(y[k][e], up, p0, p1, p2, e);
                sm->limb[0][g] = (int)p0; sm->limb[1][g] = (int)p1; sm->limb[2][g] = (int)p2;
            }
        }
        consumers_sync();
    }
    return out;
}

// Row sums of R rows held per lane, reduced over the warp with R-way transposed
// butterflies (R = 1, 2: 5 shuffles; R = 3, 4: 6).  Lane L ends with the full
// sum of row L >> 4 (R = 2) or L >> 3 (R = 3, 4); any lane for R = 1.
template <int R>
__device__ __forceinline__ float xreduce(const float (&v)[R], int lane) {
    if constexpr (R == 1) {
        return warp_sum(v[0]);
    } else if constexpr (R == 2) {
        const bool hi = lane & 16;
        float k = hi ? v[1] : v[0];
        const float s = hi ? v[0] : v[1];
        k += __shfl_xor_sync(0xffffffffu, s, 16);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) k += __shfl_xor_sync(0xffffffffu, k, o);
        return k;
    } else {
        static_assert(R == 3 || R == 4, "");
        const float v3 = R == 4 ? v[R - 1] : 0.f;
        const bool hi = lane & 16;
        float k0 = hi ? v[2] : v[0], k1 = hi ? v3 : v[1];
        const float s0 = hi ? v[0] : v[2], s1 = hi ? v[1] : v3;
        k0 += __shfl_xor_sync(0xffffffffu, s0, 16);
        k1 += __shfl_xor_sync(0xffffffffu, s1, 16);
        const bool h8 = lane & 8;
        float k = h8 ? k1 : k0;
        const float s = h8 ? k0 : k1;
        k += __shfl_xor_sync(0xffffffffu, s, 8);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) k += __shfl_xor_sync(0xffffffffu, k, o);
        return k;
    }
}
// a2 * 2^16 + a1 * 2^8 + a0 in fp32 (a1 * 256 + a0 fits int32; one rounding in the fma).
__device__ __forceinline__ float limb_sum_f32(int a0, int a1, int a2) {
    return fmaf((float)a2, 65536.f, (float)(a1 * 256 + a0));
}

// INT8 matvec over rows [r0, r1) of one projection (K wide) on the limbs the
// gather left in shared memory.  The phase's chunks (MAXCH at most) are taken
// together; warp w handles rows w, w + NCW, ... (RMAX at most) at once, so the
// loads and dp4a chains of its rows overlap and one transposed reduction ends
// them.  out(row, dot * 2^-k * scl(row)) is called once per row.
template <int K, int RMAX, int MAXCH, class Scl, class Out>
MQ_PHASE void mv_rows8(Ctx& c, Cons& cs, int r0, int r1, float inv, Scl scl, Out out) {
    constexpr int RS = K + ROW_SKEW;
    constexpr int RPC = STAGE_BYTES / RS;
    constexpr int UPL = K / 512;
    const int n = r1 - r0;
    const int nch = (n + RPC - 1) / RPC;
    Limbs<UPL * 4> lb;
    lb.load(cs.sm->limb[0], cs.sm->limb[1], cs.sm->limb[2], cs.lane, inv);
    const uint8_t* st[MAXCH];
#pragma unroll
    for (int q = 0; q < MAXCH; ++q) st[q] = q < nch ? cs.wait_at(c, q, 1) : nullptr;
    int acc[RMAX][3];
    const uint4* rowp[RMAX];
#pragma unroll
    for (int r = 0; r < RMAX; ++r) {
        acc[r][0] = acc[r][1] = acc[r][2] = 0;
        const int i = cs.warp + NCW * r;
        rowp[r] = i < n ? reinterpret_cast<const uint4*>(pick(st, i / RPC) + (size_t)(i % RPC) * RS) : nullptr;
    }
#pragma unroll
    for (int j = 0; j < UPL; ++j)
#pragma unroll
        for (int r = 0; r < RMAX; ++r)
            if (rowp[r]) lb.acc(rowp[r][cs.lane + 32 * j], j, acc[r][0], acc[r][1], acc[r][2]);
    float v[RMAX];
#pragma unroll
    for (int r = 0; r < RMAX; ++r) v[r] = limb_sum_f32(acc[r][0], acc[r][1], acc[r][2]);
    const float tot = xreduce<RMAX>(v, cs.lane);
    const int rr = RMAX == 1 ? 0 : (RMAX == 2 ? cs.lane >> 4 : cs.lane >> 3);
    const int lead = RMAX == 1 ? 0 : (RMAX == 2 ? (cs.lane & 15) : (cs.lane & 7));
    const int i = cs.warp + NCW * rr;
    if (lead == 0 && rr < RMAX && i < n) out(r0 + i, tot * inv * scl(r0 + i));
    cs.release_n(nch);
}

// gate/up pairs [p0, p1) (INT8, limbs in shared memory): warp w handles pairs
// w and w + NCW at once (4 rows); val(gate, up) -> published value.
template <int MAXCH, class Val, class Out>
MQ_PHASE void gu_rows8(Ctx& c, Cons& cs, int p0, int p1, float inv, const float* sg, const float* su, Val val,
                       Out out) {
    constexpr int K = HIDDEN;
    constexpr int RS = K + ROW_SKEW;
    constexpr int PPC = STAGE_BYTES / (2 * RS);   // pairs per chunk
    constexpr int UPL = K / 512;
    const int n = p1 - p0;
    const int nch = (n + PPC - 1) / PPC;
    Limbs<UPL * 4> lb;
    lb.load(cs.sm->limb[0], cs.sm->limb[1], cs.sm->limb[2], cs.lane, inv);
    const uint8_t* st[MAXCH];
#pragma unroll
    for (int q = 0; q < MAXCH; ++q) st[q] = q < nch ? cs.wait_at(c, q, 2) : nullptr;
    int acc[4][3];
    const uint4* rowp[4];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int i = cs.warp + NCW * r;
        const uint8_t* ch = i < n ? pick(st, i / PPC) : nullptr;
        const int q = i / PPC, nin = min(PPC, n - q * PPC);
        rowp[2 * r] = ch ? reinterpret_cast<const uint4*>(ch + (size_t)(i - q * PPC) * RS) : nullptr;
        rowp[2 * r + 1] = ch ? reinterpret_cast<const uint4*>(ch + (size_t)(nin + i - q * PPC) * RS) : nullptr;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[r][0] = acc[r][1] = acc[r][2] = 0;
#pragma unroll
    for (int j = 0; j < UPL; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r)
            if (rowp[r]) lb.acc(rowp[r][cs.lane + 32 * j], j, acc[r][0], acc[r][1], acc[r][2]);
    float v[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) v[r] = limb_sum_f32(acc[r][0], acc[r][1], acc[r][2]);
    const float tot = xreduce<4>(v, cs.lane);          // lane 8 m + {0..7}: row m = (g0, u0, g1, u1)
    const float upv = __shfl_down_sync(0xffffffffu, tot, 8);
    const int i = cs.warp + NCW * (cs.lane >> 4);
    if ((cs.lane & 15) == 0 && i < n) out(p0 + i, val(tot * inv * sg[i], upv * inv * su[i]));
    cs.release_n(nch);
}

__device__ __forceinline__ uint32_t tag_of(uint32_t epoch, int layer, int e) {
    return epoch + 1u + (uint32_t)layer * TAGS_PER_LAYER + (uint32_t)e;
}
enum { E_H = 0, E_QKV = 1, E_PART = 2, E_ATTN = 3, E_ACT = 4, E_MLP = 5 };


// ---------------------------------------------------------------------------
// Attention for one (KV head g, position split s) item.
// ---------------------------------------------------------------------------
// QK RMSNorm over one 128-wide head then split-half RoPE at the current position
// (a10_int8_decode_kernel.cu:160-192, int8_decoder.py:234-240).  Lane holds
// dims lane + 32j, so the RoPE partners (i, i+64) are j and j+2 of one lane.
// Norm weights and the cos/sin row are loaded ahead of the exchange wait.
// The weights and the cos/sin row are kept as raw bf16 bits until use: converting
// them at load time would stall the warp on the loads before its exchange poll.
struct RopeRegs {
    uint16_t nw[4], cs[4], sn[4];
    __device__ __forceinline__ void load(const void* normw, const __nv_bfloat16* cosr, const __nv_bfloat16* sinr,
                                         int lane) {
        const uint16_t* w = (const uint16_t*)normw;
        const uint16_t* cr = (const uint16_t*)cosr;
        const uint16_t* sr = (const uint16_t*)sinr;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            nw[j] = __ldg(w + lane + 32 * j);
            cs[j] = __ldg(cr + lane + 32 * j);
            sn[j] = __ldg(sr + lane + 32 * j);
        }
    }
};
__device__ __forceinline__ void qk_norm_rope(const float* raw, const RopeRegs& R, int lane, float out[4]) {
    float v[4];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) { v[j] = raw[lane + 32 * j]; ss += v[j] * v[j]; }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)HD + RMS_EPS);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = v[j] * r * bf16_bits_to_f32(R.nw[j]);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const float c0 = bf16_bits_to_f32(R.cs[j]), s0 = bf16_bits_to_f32(R.sn[j]);
        const float c2 = bf16_bits_to_f32(R.cs[j + 2]), s2 = bf16_bits_to_f32(R.sn[j + 2]);
        out[j] = v[j] * c0 - v[j + 2] * s0;
        out[j + 2] = v[j] * s2 + v[j + 2] * c2;
    }
}

// Splits with at most this many cached positions take the one-position-per-warp
// path (measured: the attention phase at position 10 drops from 2.8 to 1.8 us; at
// 60 positions both paths cost the same, at 200 the chunk path is faster).
constexpr int SHORT_SPLIT = 96;

MQ_PHASE void attention_item(const DecodeParams& P, Ctx& c, Cons& cs, const Geo& G, int l, uint32_t epoch) {
    Smem* sm = cs.sm;
    const int par = l & 1;
    const uint32_t tq = tag_of(epoch, l, E_QKV);
    const int pos = G.c - 1;
    RopeRegs R;
    if (cs.warp < 3)  // warps 0,1: q heads (q_norm); warp 2: k head (k_norm)
        R.load(sm->lw[l][cs.warp < 2 ? 4 : 5], P.cos_t + (size_t)pos * HD, P.sin_t + (size_t)pos * HD, cs.lane);
    // raw q (two heads), k, v of KV head g: three runs of the q|k|v row space, one gathered poll
    {
        const uint64_t* xq = c.ws->xqkv[par];
        const int g = G.g;
        uint32_t pay[1][4];
        poll_groups_at<1>(c, cs, [&](int gr) {
            const int i = 4 * gr;   // the three runs are 4-word aligned
            return xq + (i < 2 * HD ? 2 * g * HD + i
                                    : (i < 3 * HD ? QSZ + g * HD + (i - 2 * HD) : QSZ + KVSZ + g * HD + (i - 3 * HD)));
        }, HD, tq, 10, pay);
        if (cs.tid < HD)
            *reinterpret_cast<float4*>(sm->raw + 4 * cs.tid) = make_float4(
                __uint_as_float(pay[0][0]), __uint_as_float(pay[0][1]), __uint_as_float(pay[0][2]), __uint_as_float(pay[0][3]));
    }
    consumers_sync();
    if (cs.warp < 2) {
        float o[4];
        qk_norm_rope(sm->raw + cs.warp * HD, R, cs.lane, o);
#pragma unroll
        for (int j = 0; j < 4; ++j) sm->q[cs.warp][cs.lane + 32 * j] = o[j];
    } else if (cs.warp == 2 && G.owner) {
        float o[4];
        qk_norm_rope(sm->raw + 2 * HD, R, cs.lane, o);
        const size_t off = (((size_t)l * NKVH + G.g) * (size_t)P.max_seq + pos) * HD;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = cs.lane + 32 * j;
            const uint16_t kb = (uint16_t)f32_to_bf16_bits(o[j]);
            const uint16_t vb = (uint16_t)f32_to_bf16_bits(sm->raw[3 * HD + i]);
            sm->kvcur[0][i] = kb;
            sm->kvcur[1][i] = vb;
            reinterpret_cast<uint16_t*>(P.kc)[off + i] = kb;
            reinterpret_cast<uint16_t*>(P.vc)[off + i] = vb;
        }
    }
    consumers_sync();
    // Flash-decode inside the CTA without block barriers.  On long splits warp w owns
    // the ring chunks (32 positions each) that land in stages s with s % NCW == w and
    // keeps its own online-softmax state (m, l, acc) for both GQA heads.  Within a
    // chunk lane (g, h) scores positions 2g, 2g+1 over dims 64h .. 64h+63 (dims
    // visited in a lane-rotated order so the lanes hit different banks), one
    // max/sum reduction per chunk, and P.V is accumulated with lane holding dims
    // 4*lane .. 4*lane+3.
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
    const float scale = P.attn_scale;
    const float4* q0v = reinterpret_cast<const float4*>(sm->q[0]);
    const float4* q1v = reinterpret_cast<const float4*>(sm->q[1]);
    auto chunk = [&](const uint16_t* kb, const uint16_t* vb, int n) {
        // Lane (g, h) = (lane % 16, lane / 16) scores positions 2g and 2g+1 over dims
        // 64h .. 64h+63 (one q load serves two positions); one shuffle joins the halves.
        const int g = cs.lane & 15, dh = cs.lane >> 4;
        const int pa = 2 * g, pb = pa + 1;
        float sa0 = -INFINITY, sa1 = -INFINITY, sb0 = -INFINITY, sb1 = -INFINITY;
        {
            const uint16_t* ka = kb + (pa < n ? pa : 0) * HD + dh * (HD / 2);
            const uint16_t* kc = kb + (pb < n ? pb : 0) * HD + dh * (HD / 2);
            const float4* qa = q0v + dh * (HD / 8);
            const float4* qb = q1v + dh * (HD / 8);
            float xa = 0.f, xb = 0.f, ya = 0.f, yb = 0.f, xa2 = 0.f, xb2 = 0.f, ya2 = 0.f, yb2 = 0.f;
#pragma unroll 8
            for (int i = 0; i < HD / 8; ++i) {
                const int d4 = (g + i) & (HD / 8 - 1);
                const uint2 wa = *reinterpret_cast<const uint2*>(ka + 4 * d4);
                const uint2 wb = *reinterpret_cast<const uint2*>(kc + 4 * d4);
                const float4 q0 = qa[d4], q1 = qb[d4];
                const float a0 = bf16_bits_to_f32(wa.x & 0xffffu), a1 = bf16_bits_to_f32(wa.x >> 16);
                const float a2 = bf16_bits_to_f32(wa.y & 0xffffu), a3 = bf16_bits_to_f32(wa.y >> 16);
                const float b0 = bf16_bits_to_f32(wb.x & 0xffffu), b1 = bf16_bits_to_f32(wb.x >> 16);
                const float b2 = bf16_bits_to_f32(wb.y & 0xffffu), b3 = bf16_bits_to_f32(wb.y >> 16);
                xa = fmaf(q0.x, a0, xa); xa2 = fmaf(q0.y, a1, xa2); xa = fmaf(q0.z, a2, xa); xa2 = fmaf(q0.w, a3, xa2);
                ya = fmaf(q1.x, a0, ya); ya2 = fmaf(q1.y, a1, ya2); ya = fmaf(q1.z, a2, ya); ya2 = fmaf(q1.w, a3, ya2);
                xb = fmaf(q0.x, b0, xb); xb2 = fmaf(q0.y, b1, xb2); xb = fmaf(q0.z, b2, xb); xb2 = fmaf(q0.w, b3, xb2);
                yb = fmaf(q1.x, b0, yb); yb2 = fmaf(q1.y, b1, yb2); yb = fmaf(q1.z, b2, yb); yb2 = fmaf(q1.w, b3, yb2);
            }
            xa += xa2; ya += ya2; xb += xb2; yb += yb2;
            xa += __shfl_xor_sync(0xffffffffu, xa, 16);
            ya += __shfl_xor_sync(0xffffffffu, ya, 16);
            xb += __shfl_xor_sync(0xffffffffu, xb, 16);
            yb += __shfl_xor_sync(0xffffffffu, yb, 16);
            if (pa < n) { sa0 = xa * scale; sa1 = ya * scale; }
            if (pb < n) { sb0 = xb * scale; sb1 = yb * scale; }
        }
        const float n0 = fmaxf(m0, warp_max(fmaxf(sa0, sb0))), n1 = fmaxf(m1, warp_max(fmaxf(sa1, sb1)));
        const float c0 = expf(m0 - n0), c1 = expf(m1 - n1);   // 0 while m is still -inf
        const float ea0 = pa < n ? expf(sa0 - n0) : 0.f, eb0 = pb < n ? expf(sb0 - n0) : 0.f;
        const float ea1 = pa < n ? expf(sa1 - n1) : 0.f, eb1 = pb < n ? expf(sb1 - n1) : 0.f;
        // lanes g and g + 16 hold the same weights: sum one half only
        l0 = l0 * c0 + warp_sum(dh ? 0.f : ea0 + eb0);
        l1 = l1 * c1 + warp_sum(dh ? 0.f : ea1 + eb1);
#pragma unroll
        for (int j = 0; j < 4; ++j) { a0[j] *= c0; a1[j] *= c1; }
        auto pv = [&](int p) {
            const float ep0 = __shfl_sync(0xffffffffu, (p & 1) ? eb0 : ea0, p >> 1);
            const float ep1 = __shfl_sync(0xffffffffu, (p & 1) ? eb1 : ea1, p >> 1);
            const uint2 vw = *reinterpret_cast<const uint2*>(vb + p * HD + 4 * cs.lane);
            const float v0 = bf16_bits_to_f32(vw.x & 0xffffu), v1 = bf16_bits_to_f32(vw.x >> 16);
            const float v2 = bf16_bits_to_f32(vw.y & 0xffffu), v3 = bf16_bits_to_f32(vw.y >> 16);
            a0[0] = fmaf(ep0, v0, a0[0]); a0[1] = fmaf(ep0, v1, a0[1]); a0[2] = fmaf(ep0, v2, a0[2]); a0[3] = fmaf(ep0, v3, a0[3]);
            a1[0] = fmaf(ep1, v0, a1[0]); a1[1] = fmaf(ep1, v1, a1[1]); a1[2] = fmaf(ep1, v2, a1[2]); a1[3] = fmaf(ep1, v3, a1[3]);
        };
        if (n == KV_CHUNK_POS) {   // full chunk: constant trip count, so loads and shuffles overlap
#pragma unroll 8
            for (int p = 0; p < KV_CHUNK_POS; ++p) pv(p);
        } else {
            for (int p = 0; p < n; ++p) pv(p);
        }
        m0 = n0;
        m1 = n1;
    };
    if (G.past1 - G.past0 <= SHORT_SPLIT) {
        // Short split: one position per warp at a time, all NCW warps busy (a whole chunk
        // on one warp would leave the others idle).  Lane L holds dims 4L .. 4L+3 of both q
        // heads; a position costs one 8-byte K and V load per lane and two warp sums.
        const float4 q0r = q0v[cs.lane], q1r = q1v[cs.lane];
        auto one = [&](const uint16_t* kr, const uint16_t* vr) {
            const uint2 kw = *reinterpret_cast<const uint2*>(kr + 4 * cs.lane);
            const uint2 vw = *reinterpret_cast<const uint2*>(vr + 4 * cs.lane);
            const float k0 = bf16_bits_to_f32(kw.x & 0xffffu), k1 = bf16_bits_to_f32(kw.x >> 16);
            const float k2 = bf16_bits_to_f32(kw.y & 0xffffu), k3 = bf16_bits_to_f32(kw.y >> 16);
            float x = fmaf(q0r.x, k0, fmaf(q0r.y, k1, fmaf(q0r.z, k2, q0r.w * k3)));
            float y = fmaf(q1r.x, k0, fmaf(q1r.y, k1, fmaf(q1r.z, k2, q1r.w * k3)));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                x += __shfl_xor_sync(0xffffffffu, x, o);
                y += __shfl_xor_sync(0xffffffffu, y, o);
            }
            const float s0 = x * scale, s1 = y * scale;
            const float n0 = fmaxf(m0, s0), n1 = fmaxf(m1, s1);
            const float c0 = expf(m0 - n0), c1 = expf(m1 - n1);   // 0 while m is still -inf
            const float e0 = expf(s0 - n0), e1 = expf(s1 - n1);
            l0 = l0 * c0 + e0;
            l1 = l1 * c1 + e1;
            const float v[4] = {bf16_bits_to_f32(vw.x & 0xffffu), bf16_bits_to_f32(vw.x >> 16),
                                bf16_bits_to_f32(vw.y & 0xffffu), bf16_bits_to_f32(vw.y >> 16)};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                a0[j] = fmaf(e0, v[j], a0[j] * c0);
                a1[j] = fmaf(e1, v[j], a1[j] * c1);
            }
            m0 = n0;
            m1 = n1;
        };
        int base = 0;   // item-relative index of the chunk's first position
        for (int p = G.past0; p < G.past1; p += KV_CHUNK_POS, base += KV_CHUNK_POS) {
            const int n = min(KV_CHUNK_POS, G.past1 - p);
            const uint16_t* kb = reinterpret_cast<const uint16_t*>(cs.wait(c, 3));
            const uint16_t* vb = kb + KV_V_OFFSET / 2;
            for (int i = (cs.warp - base % NCW + NCW) % NCW; i < n; i += NCW) one(kb + i * HD, vb + i * HD);
            cs.release();
        }
        if (G.owner && (G.past1 - G.past0) % NCW == cs.warp) one(sm->kvcur[0], sm->kvcur[1]);   // the current position
    } else {
        // Warp (stage % NCW) alone reads the chunks of a ring stage here, so a stage is
        // free as soon as that warp is done with it, whatever the other warps are doing.
        for (int p = G.past0; p < G.past1; p += KV_CHUNK_POS) {
            const int n = min(KV_CHUNK_POS, G.past1 - p);
            if ((int)(cs.seq % NSTAGE) % NCW == cs.warp) {
                const uint8_t* st = cs.wait(c, 3);
                chunk(reinterpret_cast<const uint16_t*>(st), reinterpret_cast<const uint16_t*>(st + KV_V_OFFSET), n);
                cs.release_owned();
            } else {
                cs.skip();
            }
        }
        if (G.owner && cs.warp == NCW - 1) chunk(sm->kvcur[0], sm->kvcur[1], 1);  // the current position
    }
    // Merge the NCW warp states through shared memory (x is free during attention).
    float* wacc = sm->x;  // [NCW][2][HD]
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        wacc[(cs.warp * 2 + 0) * HD + 4 * cs.lane + j] = a0[j];
        wacc[(cs.warp * 2 + 1) * HD + 4 * cs.lane + j] = a1[j];
    }
    if (cs.lane == 0) {
        sm->sc[0][cs.warp] = m0; sm->sc[1][cs.warp] = m1;
        sm->pe[0][cs.warp] = l0; sm->pe[1][cs.warp] = l1;
    }
    consumers_sync();
    float acc = 0.f, M = -INFINITY, L = 0.f;
    if (cs.tid < 2 * HD) {
        const int h = cs.tid >> 7, d = cs.tid & (HD - 1);
#pragma unroll
        for (int w = 0; w < NCW; ++w) M = fmaxf(M, sm->sc[h][w]);
#pragma unroll
        for (int w = 0; w < NCW; ++w) {
            const float e = expf(sm->sc[h][w] - M);  // 0 for a warp that saw no position
            L = fmaf(sm->pe[h][w], e, L);
            acc = fmaf(wacc[(w * 2 + h) * HD + d], e, acc);
        }
    }
    if (G.S == 1) {
        if (cs.tid < 2 * HD)
            st_tagged(&c.ws->xattn[par][G.g * 2 * HD + cs.tid], tag_of(epoch, l, E_ATTN), __float_as_uint(acc / L));
        return;
    }
    // Split-K: publish (acc, m, l), then merge this split's slice of the pair's 256 outputs.
    const uint32_t tp = tag_of(epoch, l, E_PART);
    uint64_t* part = c.ws->xpart[par];
    if (cs.tid < 2 * HD) {
        st_tagged(&part[G.item * PART_WORDS + cs.tid], tp, __float_as_uint(acc));
        if ((cs.tid & (HD - 1)) == 0) {
            const int h = cs.tid >> 7;
            st_tagged(&part[G.item * PART_WORDS + 2 * HD + h], tp, __float_as_uint(M));
            st_tagged(&part[G.item * PART_WORDS + 2 * HD + 2 + h], tp, __float_as_uint(L));
        }
    }
    const int j0 = split_lo(2 * HD, G.S, G.s), j1 = split_lo(2 * HD, G.S, G.s + 1);
    const int nj = j1 - j0;   // this split's slice of the pair's 256 outputs (nj * S <= 256 + S threads)
    const int base_item = G.g * G.S;
    // All the slice's tagged words in one round: thread k < nj * S reads acc[split t][j0 + jj],
    // threads k < 4 S the (m, l) of (split, head); then one merge per output from shared memory.
    consumers_sync();   // x (the warp-merge buffer) and raw are free again
    float* sa = sm->x;    // [S][nj]
    float* sml = sm->raw; // [S][4]: m0, m1, l0, l1
    if (cs.tid < nj * G.S) {
        const int t = cs.tid / nj, jj = cs.tid - t * nj;
        sa[t * nj + jj] = __uint_as_float(poll_word(c, &part[(base_item + t) * PART_WORDS + j0 + jj], tp, 12));
    }
    if (cs.tid < 4 * G.S) {
        const int t = cs.tid >> 2, q = cs.tid & 3;
        sml[t * 4 + q] = __uint_as_float(poll_word(c, &part[(base_item + t) * PART_WORDS + 2 * HD + q], tp, 11));
    }
    consumers_sync();
    if (cs.tid < nj) {
        const int j = j0 + cs.tid, h = j >> 7;
        float M = -INFINITY, L = 0.f, o = 0.f;
        for (int t = 0; t < G.S; ++t) {
            const float mt = sml[t * 4 + h], lt = sml[t * 4 + 2 + h], at = sa[t * nj + cs.tid];
            const float Mn = fmaxf(M, mt);
            const float cp = expf(M - Mn), ct = expf(mt - Mn);
            L = L * cp + lt * ct;
            o = o * cp + at * ct;
            M = Mn;
        }
        st_tagged(&c.ws->xattn[par][G.g * 2 * HD + j], tag_of(epoch, l, E_ATTN), __float_as_uint(o / L));
    }
}


// ---------------------------------------------------------------------------
// Consumer main: the layer loop.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void trace_stamp(const DecodeParams& P, const Cons& cs, int slot) {
    if (P.trace && cs.tid == 0 && slot < P.trace_slots)
        P.trace[(size_t)blockIdx.x * P.trace_slots + slot] = globaltimer();
}

enum { LW_IN = 0, LW_Q, LW_K, LW_V, LW_QN, LW_KN, LW_O, LW_POST, LW_G, LW_U, LW_D };
enum { LS_Q = 0, LS_K, LS_V, LS_O, LS_G, LS_U, LS_D };

// Pointer tables of every layer into shared memory (one dependent global load
// per pointer at kernel start instead of one per phase).
__device__ __forceinline__ void stage_pointers(const DecodeParams& P, const Cons& cs, bool scaled) {
    const int per = scaled ? 18 : 11;
    constexpr int MAXI = (MAX_LAYERS * 18 + NCT - 1) / NCT;
    const void* v[MAXI];
#pragma unroll
    for (int k = 0; k < MAXI; ++k) {   // all loads first, so they are in flight together
        const int i = cs.tid + k * NCT;
        v[k] = nullptr;
        if (i < P.L * per) {
            const int l = i / per, f = i % per;
            v[k] = f < 11 ? reinterpret_cast<const void* const*>(&P.layers[l])[f]
                          : reinterpret_cast<const void* const*>(&P.scales[l])[f - 11];
        }
    }
#pragma unroll
    for (int k = 0; k < MAXI; ++k) {
        const int i = cs.tid + k * NCT;
        if (i < P.L * per) {
            const int l = i / per, f = i % per;
            if (f < 11) cs.sm->lw[l][f] = v[k];
            else cs.sm->ls[l][f - 11] = reinterpret_cast<const float*>(v[k]);
        }
    }
}

// Every per-row scale this CTA will need in the step, into shared memory, so
// that no matvec row waits on a dependent global load.  Needs the staged
// pointer tables (call after stage_pointers + a consumer barrier).  Each thread
// issues all of its loads before it stores any, so their latencies overlap.
__device__ __forceinline__ void stage_scales(const DecodeParams& P, const Cons& cs, const Geo& G) {
    Smem* sm = cs.sm;
    constexpr int MAXI = (MAX_LAYERS * SCL_STRIDE + NCT - 1) / NCT;
    constexpr int MAXJ = (LM_MAXR + NCT - 1) / NCT;
    float v[MAXI], w[MAXJ];
#pragma unroll
    for (int k = 0; k < MAXI; ++k) {
        const int i = cs.tid + k * NCT;
        const float* src = nullptr;
        if (i < P.L * SCL_STRIDE) {
            const int l = i / SCL_STRIDE, j = i % SCL_STRIDE;
            if (j < SCL_O) {
                const int r = G.qkv0 + j;
                if (r < G.qkv1)
                    src = r < QSZ ? sm->ls[l][LS_Q] + r
                                  : (r < QSZ + KVSZ ? sm->ls[l][LS_K] + (r - QSZ) : sm->ls[l][LS_V] + (r - QSZ - KVSZ));
            } else if (j < SCL_G) {
                const int r = G.o0 + (j - SCL_O);
                if (r < G.o1) src = sm->ls[l][LS_O] + r;
            } else if (j < SCL_U) {
                const int r = G.gu0 + (j - SCL_G);
                if (r < G.gu1) src = sm->ls[l][LS_G] + r;
            } else if (j < SCL_D) {
                const int r = G.gu0 + (j - SCL_U);
                if (r < G.gu1) src = sm->ls[l][LS_U] + r;
            } else {
                const int r = G.d0 + (j - SCL_D);
                if (r < G.d1) src = sm->ls[l][LS_D] + r;
            }
        }
        v[k] = src ? __ldg(src) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < MAXJ; ++k) {
        const int j = cs.tid + k * NCT;
        w[k] = j < G.lm1 - G.lm0 ? __ldg(P.lm_scale + G.lm0 + j) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < MAXI; ++k) {
        const int i = cs.tid + k * NCT;
        if (i < P.L * SCL_STRIDE) sm->scl[i] = v[k];
    }
#pragma unroll
    for (int k = 0; k < MAXJ; ++k) {
        const int j = cs.tid + k * NCT;
        if (j < G.lm1 - G.lm0) sm->lm_scl[j] = w[k];
    }
}

template <class WT>
__device__ void consumer_main(const DecodeParams& P, Ctx& c, const Geo& G, uint32_t& epoch,
                              unsigned long long& cta_key) {
    constexpr bool L8 = WT::LIMBS;
    Smem* sm = c.sm;
    Cons cs{sm, 0u, (int)(threadIdx.x >> 5), (int)(threadIdx.x & 31), (int)threadIdx.x};
    Workspace* ws = c.ws;
    const bool cta0 = G.b == 0;
    stage_pointers(P, cs, WT::HAS_SCALE);
    for (int i = cs.tid; i < INTER / 4; i += NCT) sm->limb[3][i] = 0;   // zero B columns of the LM-head mma
    consumers_sync();
    if (WT::HAS_SCALE) stage_scales(P, cs, G);
    NormW4 w_in, w_post;
    w_in.load(cs, sm->lw[0][LW_IN]);
    // Everything below reads what the previous step wrote (epoch, input token,
    // hand-off words, KV cache); everything above reads only weights and tables.
    pdl_wait();
    epoch = ld_relaxed32(&P.ws->epoch);
    int token = P.token_in_dev ? *(volatile const int*)P.token_in_dev : P.token_in;
    if (token < 0 || token >= VOCAB) {
        if (cs.tid == 0) {
            if (cta0) record_error(c, MQ_DEV_BAD_TOKEN, token);
            sm->abort_flag = 1;
        }
        token = 0;
    }
    consumers_sync();
    InputScale xin{1.f, 1.f};
    {   // layer-0 input: the embedding row (no exchange)
        uint32_t pay[1][4] = {{0u, 0u, 0u, 0u}};
        if (cs.tid < HIDDEN / 4 && !*(volatile int*)&sm->abort_flag) {
            const uint2 u = __ldg(reinterpret_cast<const uint2*>((const __nv_bfloat16*)P.embed + (size_t)token * HIDDEN) + cs.tid);
            pay[0][0] = u.x & 0xffffu; pay[0][1] = u.x >> 16; pay[0][2] = u.y & 0xffffu; pay[0][3] = u.y >> 16;
        }
        xin = finish_input<1, L8, true>(cs, pay, HIDDEN / 4, true, w_in, sm->x, sm->h);
    }
    for (int l = 0; l < P.L; ++l) {
        const int par = l & 1;
        const int tb = l * TRACE_PER_LAYER;
        if (l > 0) {
            if (consumers_sync_abort(c)) break;
            uint32_t pay[1][4];
            poll_groups<1>(c, cs, ws->xh[par], HIDDEN / 4, tag_of(epoch, l, E_H), 20, pay);
            if (cta0 && P.layer_hidden && cs.tid < HIDDEN / 4) {
                float* lh = P.layer_hidden + (size_t)(l - 1) * HIDDEN + 4 * cs.tid;
                for (int e = 0; e < 4; ++e) lh[e] = bf16_bits_to_f32(pay[0][e] & 0xffffu);
            }
            xin = finish_input<1, L8, true>(cs, pay, HIDDEN / 4, true, w_in, sm->x, sm->h);
        }
        trace_stamp(P, cs, tb + TR_START);
        w_post.load(cs, sm->lw[l][LW_POST]);  // needed after attention: its latency is hidden
        const float* lsc = sm->scl + l * SCL_STRIDE;
        // --- QKV ---
        {
            const uint32_t t = tag_of(epoch, l, E_QKV);
            const bool skip = (l == 0 && G.b == P.skip_cta);
            uint64_t* dst = ws->xqkv[par];
            const float rstd = xin.rstd;
            auto scl = [&](int r) { return (WT::HAS_SCALE ? lsc[r - G.qkv0] : 1.f) * rstd; };
            auto out = [&](int r, float d) {
                if (!skip) st_tagged(&dst[r], t, __float_as_uint(d));
            };
            if constexpr (L8) mv_rows8<HIDDEN, 3, 2>(c, cs, G.qkv0, G.qkv1, xin.inv, scl, out);
            else mv_phase<WT, HIDDEN>(c, cs, G.qkv0, G.qkv1, sm->x, scl, out);
        }
        trace_stamp(P, cs, tb + TR_QKV);
        // --- attention (only CTAs that own an item) ---
        if (G.item >= 0) {
            if (consumers_sync_abort(c)) break;
            attention_item(P, c, cs, G, l, epoch);
            trace_stamp(P, cs, tb + TR_ATTN);
        }
        // --- O projection + residual ---
        if (consumers_sync_abort(c)) break;
        {
            uint32_t pay[2][4];
            poll_groups<2>(c, cs, ws->xattn[par], QSZ / 4, tag_of(epoch, l, E_ATTN), 30, pay);
            const NormW4 one{};
            xin = finish_input<2, L8, false>(cs, pay, QSZ / 4, false, one, sm->x, nullptr);
        }
        trace_stamp(P, cs, tb + TR_OIN);
        {
            const uint32_t t = tag_of(epoch, l, E_ACT);
            uint64_t* dst = ws->xact[par];
            auto scl = [&](int r) { return WT::HAS_SCALE ? lsc[SCL_O + r - G.o0] : 1.f; };
            auto out = [&](int r, float d) { st_tagged(&dst[r], t, __float_as_uint(d + sm->h[r])); };
            if constexpr (L8) mv_rows8<QSZ, 1, 1>(c, cs, G.o0, G.o1, xin.inv, scl, out);
            else mv_phase<WT, QSZ>(c, cs, G.o0, G.o1, sm->x, scl, out);
        }
        trace_stamp(P, cs, tb + TR_O);
        // --- post-attention norm + gate/up ---
        if (consumers_sync_abort(c)) break;
        {
            uint32_t pay[1][4];
            poll_groups<1>(c, cs, ws->xact[par], HIDDEN / 4, tag_of(epoch, l, E_ACT), 40, pay);
            xin = finish_input<1, L8, true>(cs, pay, HIDDEN / 4, false, w_post, sm->x, sm->act);
        }
        w_in.load(cs, l + 1 < P.L ? sm->lw[l + 1][LW_IN] : P.final_norm);  // next norm, loaded ahead
        trace_stamp(P, cs, tb + TR_NORM2);
        {
            const uint32_t t = tag_of(epoch, l, E_MLP);
            uint64_t* dst = ws->xmlp[par];
            const float rstd = xin.rstd;
            auto val = [&](float gd, float ud) {
                gd *= rstd;
                ud *= rstd;
                const float silu = gd / (1.0f + expf(-gd));
                return silu * ud;
            };
            auto out = [&](int r, float gd, float ud) { st_tagged(&dst[r], t, __float_as_uint(val(gd, ud))); };
            auto pubf = [&](int r, float v) { st_tagged(&dst[r], t, __float_as_uint(v)); };
            if constexpr (L8) gu_rows8<3>(c, cs, G.gu0, G.gu1, xin.inv, lsc + SCL_G, lsc + SCL_U, val, pubf);
            else gu_phase<WT>(c, cs, G.gu0, G.gu1, sm->x, lsc + SCL_G, lsc + SCL_U, out);
        }
        trace_stamp(P, cs, tb + TR_GU);
        // --- down + residual -> next h (bf16) ---
        if (consumers_sync_abort(c)) break;
        {
            uint32_t pay[2][4];
            poll_groups<2>(c, cs, ws->xmlp[par], INTER / 4, tag_of(epoch, l, E_MLP), 50, pay);
            const NormW4 one{};
            xin = finish_input<2, L8, false>(cs, pay, INTER / 4, false, one, sm->x, nullptr);
        }
        trace_stamp(P, cs, tb + TR_MLPIN);
        {
            const uint32_t t = tag_of(epoch, l + 1, E_H);
            uint64_t* dst = ws->xh[(l + 1) & 1];
            auto scl = [&](int r) { return WT::HAS_SCALE ? lsc[SCL_D + r - G.d0] : 1.f; };
            auto out = [&](int r, float d) { st_tagged(&dst[r], t, f32_to_bf16_bits(d + sm->act[r])); };
            if constexpr (L8) mv_rows8<INTER, 1, 2>(c, cs, G.d0, G.d1, xin.inv, scl, out);
            else mv_phase<WT, INTER>(c, cs, G.d0, G.d1, sm->x, scl, out);
        }
        trace_stamp(P, cs, tb + TR_DOWN);
    }
    // --- final norm + LM head + argmax ---
    cta_key = 0ull;
    if (consumers_sync_abort(c)) return;
    {
        uint32_t pay[1][4];
        poll_groups<1>(c, cs, ws->xh[P.L & 1], HIDDEN / 4, tag_of(epoch, P.L, E_H), 60, pay);
        if (cta0 && P.layer_hidden && cs.tid < HIDDEN / 4) {
            float* lh = P.layer_hidden + (size_t)(P.L - 1) * HIDDEN + 4 * cs.tid;
            for (int e = 0; e < 4; ++e) lh[e] = bf16_bits_to_f32(pay[0][e] & 0xffffu);
        }
        xin = finish_input<1, L8, true>(cs, pay, HIDDEN / 4, true, w_in, sm->x, sm->h);
    }
    trace_stamp(P, cs, P.L * TRACE_PER_LAYER + 0);
    if (cta0 && P.g_normalized)
        for (int i = cs.tid; i < HIDDEN; i += NCT) P.g_normalized[i] = sm->x[i] * xin.rstd;
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    {
        float* logits = P.logits;
        const float rstd = xin.rstd;
        auto scl = [&](int r) { return (WT::HAS_SCALE ? sm->lm_scl[r - G.lm0] : 1.f) * rstd; };
        auto out = [&](int r, float d) {
            if (logits) logits[r] = d;
            if (d > best_v || (d == best_v && r < best_i)) { best_v = d; best_i = r; }
        };
        if constexpr (L8) mma_stream<HIDDEN>(c, cs, G.lm0, G.lm1, xin.inv, scl, out);
        else mv_phase<WT, HIDDEN>(c, cs, G.lm0, G.lm1, sm->x, scl, out);
    }
    // argmax over the lanes of the warp (ties: lowest row)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
        if (ov > best_v || (ov == best_v && oi < best_i)) { best_v = ov; best_i = oi; }
    }
    if (cs.lane == 0) {
        sm->best[cs.warp] = best_i == 0x7fffffff ? 0ull
                           : (((unsigned long long)float_order_key(best_v)) << 32) | (uint32_t)(~(uint32_t)best_i);
    }
    consumers_sync();
    trace_stamp(P, cs, P.L * TRACE_PER_LAYER + 1);
    if (cs.tid == 0) {
        unsigned long long k = 0ull;
        for (int i = 0; i < NCW; ++i) k = sm->best[i] > k ? sm->best[i] : k;
        cta_key = k;
    }
}

template <class WT>
__global__ void __launch_bounds__(NTHREADS, 1) decode_kernel(const DecodeParams P) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem* sm = reinterpret_cast<Smem*>(smem_raw);
    Ctx c{sm, P.ws, P.budget_ns};
    if (P.trace && threadIdx.x == 0 && P.L * TRACE_PER_LAYER + 3 < P.trace_slots)   // kernel entry
        P.trace[(size_t)blockIdx.x * P.trace_slots + P.L * TRACE_PER_LAYER + 2] = globaltimer();
    // Let the next step's grid be scheduled: its CTAs take SMs as this grid's
    // CTAs exit.  Both griddepcontrol instructions are no-ops for a grid
    // launched without programmatic stream serialisation.
    pdl_launch_dependents();
    Geo G;
    G.init(P);
    if (threadIdx.x == 0) {
        for (int s = 0; s < NSTAGE; ++s) {
            mbar_init(&sm->full[s], 1);
            mbar_init(&sm->empty[s], NCW);
        }
        sm->abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    unsigned long long cta_key = 0ull;
    uint32_t epoch = 0u;
    if (threadIdx.x >= NCT) {
        if (threadIdx.x == NCT) producer_main<WT>(P, c, G);
    } else {
        consumer_main<WT>(P, c, G, epoch, cta_key);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        Workspace* ws = P.ws;
        if (!sm->abort_flag && cta_key) atomicMax(&ws->argmax, cta_key);
        __threadfence();
        const unsigned old = atomicAdd(&ws->exit_ctr, 1u);
        if (old == gridDim.x - 1) {
            __threadfence();
            const unsigned long long key = atomicExch(&ws->argmax, 0ull);
            const int err = atomicAdd(&ws->err_code, 0);
            *P.token_out = (err != 0 || key == 0ull) ? -1 : (int)(~(uint32_t)key);
            atomicExch(&ws->exit_ctr, 0u);
            atomicExch(&ws->epoch, epoch + (uint32_t)(P.L + 1) * TAGS_PER_LAYER);
            __threadfence();
        }
        if (P.trace && P.L * TRACE_PER_LAYER + 3 < P.trace_slots)   // CTA done
            P.trace[(size_t)blockIdx.x * P.trace_slots + P.L * TRACE_PER_LAYER + 3] = globaltimer();
    }
}

// Standalone streaming matvec with the same ring and dot code (mq_matvec).
struct MatvecParams {
    const void* W;
    const float* scale;
    const float* x;
    float* y;
    Workspace* ws;
    unsigned long long budget_ns;
    int M;
};

template <class WT, int K>
__global__ void __launch_bounds__(NTHREADS, 1) matvec_kernel(const MatvecParams P) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem* sm = reinterpret_cast<Smem*>(smem_raw);
    Ctx c{sm, P.ws, P.budget_ns};
    const int r0 = split_lo(P.M, gridDim.x, blockIdx.x), r1 = split_lo(P.M, gridDim.x, blockIdx.x + 1);
    if (threadIdx.x == 0) {
        for (int s = 0; s < NSTAGE; ++s) { mbar_init(&sm->full[s], 1); mbar_init(&sm->empty[s], NCW); }
        sm->abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i < K; i += NTHREADS) sm->x[i] = P.x[i];
    __syncthreads();
    if (threadIdx.x >= NCT) {
        if (threadIdx.x == NCT) {
            Producer pr{sm, 0, 0};
            pr.rows(c, (const uint8_t*)P.W, r0, r1, K * Bytes<WT>::ESZ);
            const uint32_t first = pr.seq > (uint32_t)NSTAGE ? pr.seq - NSTAGE : 0u;
            for (uint32_t q = first; q < pr.seq; ++q) {
                unsigned long long t0 = globaltimer();
                while (!mbar_test(&sm->full[q % NSTAGE], (q / NSTAGE) & 1))
                    if (globaltimer() - t0 > c.budget) break;
            }
        }
    } else {
        Cons cs{sm, 0u, (int)(threadIdx.x >> 5), (int)(threadIdx.x & 31), (int)threadIdx.x};
        const float* sc = P.scale;
        float* y = P.y;
        auto scl = [&](int r) { return WT::HAS_SCALE ? __ldg(sc + r) : 1.f; };
        auto out = [&](int r, float d) { y[r] = d; };
        if constexpr (WT::LIMBS) {
            build_limbs(cs, sm->x, K);
            mma_stream<K>(c, cs, r0, r1, sm->limb_inv, scl, out);
        } else {
            mv_phase<WT, K>(c, cs, r0, r1, sm->x, scl, out);
        }
    }
    __syncthreads();
}

// ===========================================================================
// Host side
// ===========================================================================
namespace {

constexpr int MAX_DEV = 64;
struct DevState {
    Workspace* ws = nullptr;
    int num_sms = 0;
    bool attr_set[4] = {false, false, false, false};
    unsigned long long epoch_used = 0;   // sum of the epoch increments of the launches since the last clear
};
DevState g_dev[MAX_DEV];
unsigned long long g_budget_ns = 2000000000ull;
int g_skip_cta = -1;
int g_pos_per_split = 256;
// L2 budget for the next layer's KV prefetch (all attention splits together);
// MQ_KV_PF_MB overrides it (0: off).
unsigned long long g_kv_pf_bytes = 32ull << 20;
unsigned long long* g_trace = nullptr;
int g_trace_slots = 0;

int dev_state(DevState** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= MAX_DEV) return MQ_ERR_DEVICE;
    DevState& d = g_dev[dev];
    if (!d.ws) {
        int sms = 0;
        if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return (int)e;
        if (sms < MIN_CTAS) return MQ_ERR_DEVICE;
        Workspace* ws = nullptr;
        if ((e = cudaMalloc(&ws, sizeof(Workspace))) != cudaSuccess) return (int)e;
        if ((e = cudaMemset(ws, 0, sizeof(Workspace))) != cudaSuccess) return (int)e;
        if ((e = cudaDeviceSynchronize()) != cudaSuccess) return (int)e;
        d.ws = ws;
        d.num_sms = sms;
        if (const char* env = getenv("MQ_POS_PER_SPLIT")) {
            int v = atoi(env);
            if (v > 0) g_pos_per_split = v;
        }
        if (const char* env = getenv("MQ_KV_PF_MB")) g_kv_pf_bytes = (unsigned long long)atoll(env) << 20;
    }
    *out = &d;
    return 0;
}

template <class K>
int ensure_smem_attr(DevState& d, int slot, K kernel) {
    if (d.attr_set[slot]) return 0;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem));
    if (e != cudaSuccess) return (int)e;
    int per_sm = 0;   // the grid is one CTA per SM: one must fit
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, NTHREADS, sizeof(Smem))) != cudaSuccess)
        return (int)e;
    if (per_sm < 1) return MQ_ERR_DEVICE;
    d.attr_set[slot] = true;
    return 0;
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

int choose_splits(int cache_len, int nb) {
    int s = (cache_len + g_pos_per_split - 1) / g_pos_per_split;
    s = s < 1 ? 1 : s;
    s = s > MAX_SPLITS ? MAX_SPLITS : s;
    while (NKVH * s > nb) --s;
    if (s > cache_len) s = cache_len;
    return s < 1 ? 1 : s;
}

// One decode step is one grid of num_sms CTAs, one per SM (ensure_smem_attr
// checks that a CTA fits), so on a device without concurrent work every CTA is
// resident -- the kernel's cross-CTA hand-offs need that; a CTA held back by
// other work shows up as a bounded-wait timeout (MQ_DEV_TIMEOUT), not a hang.
// The launch allows programmatic stream serialisation: the next step's CTAs
// take SMs as this step's CTAs exit and run their read-only prologue (pointer
// tables, per-row scales, first weight copies) before griddepcontrol.wait.
// Measured on B200: +1 to +3.5 % tok/s over a cooperative launch, with or
// without the attribute (a cooperative launch gains nothing from it).  MQ_COOPERATIVE=1
// selects the plain cooperative launch.
int g_coop = -1;
cudaError_t launch_grid(const void* fn, int grid, void** args, size_t smem, cudaStream_t stream) {
    if (g_coop < 0) g_coop = getenv("MQ_COOPERATIVE") && atoi(getenv("MQ_COOPERATIVE")) ? 1 : 0;
    if (g_coop) return cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(NTHREADS), args, smem, stream);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

int launch_step(int kind, DecodeParams& P, cudaStream_t stream) {
    DevState* d = nullptr;
    int rc = dev_state(&d);
    if (rc) return rc;
    P.ws = d->ws;
    P.budget_ns = g_budget_ns;
    P.skip_cta = g_skip_cta;
    P.trace = g_trace;
    P.trace_slots = g_trace_slots;
    g_skip_cta = -1;
    P.splits = choose_splits(P.position + 1, d->num_sms);
    // Next-layer KV prefetch only while a whole layer's KV fits the budget:
    // measured, it takes ~3 % off a step at 4K cached positions, while partial
    // prefetches at 16K / 32K compete with the weight stream and cost 3-9 %.
    P.kv_pf_pos = (unsigned long long)P.position * NKVH * 2 * HD * 2 <= g_kv_pf_bytes ? P.position : 0;
    // Tags are 32-bit epochs; every launch advances the device epoch by
    // (L + 1) * TAGS_PER_LAYER.  Clear the hand-off buffers (and the epoch) long
    // before it could wrap.  `epoch_used` sums the increments actually issued.
    const unsigned long long per_launch = (unsigned long long)(P.L + 1) * TAGS_PER_LAYER;
    if (d->epoch_used + per_launch > 0xF0000000ull) {
        cudaError_t e = cudaMemsetAsync(d->ws, 0, sizeof(Workspace), stream);
        if (e != cudaSuccess) return (int)e;
        d->epoch_used = 0;
    }
    d->epoch_used += per_launch;
    void* args[] = {&P};
    cudaError_t e;
    if (kind == 0) {
        if ((rc = ensure_smem_attr(*d, 0, decode_kernel<W8>))) return rc;
        e = launch_grid((const void*)decode_kernel<W8>, d->num_sms, args, sizeof(Smem), stream);
    } else {
        if ((rc = ensure_smem_attr(*d, 1, decode_kernel<W16>))) return rc;
        e = launch_grid((const void*)decode_kernel<W16>, d->num_sms, args, sizeof(Smem), stream);
    }
    return (int)e;
}

int check_common(const void* embed, const LayerWeights* lw, const void* fnorm, const void* lm, const void* cos_t,
                 const void* sin_t, void* kc, void* vc, int L, int position, int max_seq) {
    if (!embed || !lw || !fnorm || !lm || !cos_t || !sin_t || !kc || !vc) return MQ_ERR_ARG;
    if (!aligned16(lm) || !aligned16(kc) || !aligned16(vc) || !aligned16(embed)) return MQ_ERR_ARG;
    if (L <= 0 || max_seq <= 0) return MQ_ERR_ARG;
    if (L > MAX_LAYERS) return MQ_ERR_SIZE;
    if (position < 0 || position >= max_seq) return MQ_ERR_POSITION;
    return 0;
}

}  // namespace
}  // namespace mq

using namespace mq;

extern "C" int launch_a10_int8_decode(
    int input_token_id, int* output_token_id, const void* embed_weight, const LayerWeights* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight, const float* lm_head_scale, const void* cos_table,
    const void* sin_table, void* k_cache, void* v_cache, void* /*hidden_buffer*/, void* /*g_activations*/,
    void* /*g_residual*/, void* /*g_q*/, void* /*g_k*/, void* /*g_v*/, void* /*g_attn_out*/,
    void* /*g_mlp_intermediate*/, void* g_normalized, void* /*block_max_vals*/, void* /*block_max_idxs*/,
    int num_layers, int position, int cache_len, int max_seq_len, float attn_scale, const ScalePointers* scales,
    cudaStream_t stream) {
    int rc = check_common(embed_weight, layer_weights, final_norm_weight, lm_head_weight, cos_table, sin_table,
                          k_cache, v_cache, num_layers, position, max_seq_len);
    if (rc) return rc;
    if (!output_token_id || !lm_head_scale || !scales) return MQ_ERR_ARG;
    if (cache_len != position + 1) return MQ_ERR_POSITION;
    if (input_token_id < 0 || input_token_id >= VOCAB) return MQ_ERR_TOKEN;
    DecodeParams P{};
    P.embed = embed_weight; P.layers = layer_weights; P.scales = scales; P.final_norm = final_norm_weight;
    P.lm_w = lm_head_weight; P.lm_scale = lm_head_scale;
    P.cos_t = (const __nv_bfloat16*)cos_table; P.sin_t = (const __nv_bfloat16*)sin_table;
    P.kc = (__nv_bfloat16*)k_cache; P.vc = (__nv_bfloat16*)v_cache;
    P.g_normalized = (float*)g_normalized; P.token_out = output_token_id;
    P.token_in = input_token_id; P.L = num_layers; P.position = position; P.max_seq = max_seq_len;
    P.attn_scale = attn_scale;
    return launch_step(0, P, stream);
}

extern "C" int launch_a10_decode(
    int input_token_id, int* output_token_id, const void* embed_weight, const LayerWeights* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight, const void* cos_table, const void* sin_table,
    void* k_cache, void* v_cache, void* /*hidden_buffer*/, void* /*g_activations*/, void* /*g_residual*/,
    void* /*g_q*/, void* /*g_k*/, void* /*g_v*/, void* /*g_attn_out*/, void* /*g_mlp_intermediate*/,
    void* g_normalized, void* /*block_max_vals*/, void* /*block_max_idxs*/, int num_layers, int position,
    int cache_len, int max_seq_len, float attn_scale, cudaStream_t stream) {
    int rc = check_common(embed_weight, layer_weights, final_norm_weight, lm_head_weight, cos_table, sin_table,
                          k_cache, v_cache, num_layers, position, max_seq_len);
    if (rc) return rc;
    if (!output_token_id) return MQ_ERR_ARG;
    if (cache_len != position + 1) return MQ_ERR_POSITION;
    if (input_token_id < 0 || input_token_id >= VOCAB) return MQ_ERR_TOKEN;
    DecodeParams P{};
    P.embed = embed_weight; P.layers = layer_weights; P.final_norm = final_norm_weight; P.lm_w = lm_head_weight;
    P.cos_t = (const __nv_bfloat16*)cos_table; P.sin_t = (const __nv_bfloat16*)sin_table;
    P.kc = (__nv_bfloat16*)k_cache; P.vc = (__nv_bfloat16*)v_cache;
    P.g_normalized = (float*)g_normalized; P.token_out = output_token_id;
    P.token_in = input_token_id; P.L = num_layers; P.position = position; P.max_seq = max_seq_len;
    P.attn_scale = attn_scale;
    return launch_step(1, P, stream);
}

extern "C" int mq_decode_multi(int weight_kind, int input_token, const int* d_token_in, int* d_tokens_out, int num_steps,
                               const void* embed_weight, const LayerWeights* layer_weights,
                               const void* final_norm_weight, const void* lm_head_weight,
                               const float* lm_head_scale, const ScalePointers* scales, const void* cos_table,
                               const void* sin_table, void* k_cache, void* v_cache, float* g_normalized,
                               float* d_logits, float* d_layer_hidden, int num_layers, int position,
                               int max_seq_len, float attn_scale, int row_pad_bytes, cudaStream_t stream) {
    if (weight_kind != 0 && weight_kind != 1) return MQ_ERR_ARG;
    if (!d_tokens_out || num_steps <= 0) return MQ_ERR_ARG;
    if (row_pad_bytes != 0 && row_pad_bytes != ROW_SKEW) return MQ_ERR_ARG;
    if (!d_token_in && (input_token < 0 || input_token >= VOCAB)) return MQ_ERR_TOKEN;
    int rc = check_common(embed_weight, layer_weights, final_norm_weight, lm_head_weight, cos_table, sin_table,
                          k_cache, v_cache, num_layers, position, max_seq_len);
    if (rc) return rc;
    if (position + num_steps > max_seq_len) return MQ_ERR_POSITION;
    if (weight_kind == 0 && (!lm_head_scale || !scales)) return MQ_ERR_ARG;
    for (int j = 0; j < num_steps; ++j) {
        DecodeParams P{};
        P.embed = embed_weight; P.layers = layer_weights; P.scales = scales; P.final_norm = final_norm_weight;
        P.lm_w = lm_head_weight; P.lm_scale = lm_head_scale;
        P.cos_t = (const __nv_bfloat16*)cos_table; P.sin_t = (const __nv_bfloat16*)sin_table;
        P.kc = (__nv_bfloat16*)k_cache; P.vc = (__nv_bfloat16*)v_cache;
        const bool last = j == num_steps - 1;
        P.g_normalized = last ? g_normalized : nullptr;
        P.logits = last ? d_logits : nullptr;
        P.layer_hidden = last ? d_layer_hidden : nullptr;
        P.token_in_dev = j == 0 ? d_token_in : d_tokens_out + (j - 1);
        P.token_in = input_token;
        P.row_pad = row_pad_bytes;
        P.token_out = d_tokens_out + j;
        P.L = num_layers; P.position = position + j; P.max_seq = max_seq_len; P.attn_scale = attn_scale;
        if ((rc = launch_step(weight_kind, P, stream))) return rc;
    }
    return 0;
}

extern "C" int mq_decode_step_host(const MQStepPlan* plan, int input_token, int position, cudaStream_t stream,
                                   int* out_token) {
    if (!plan || !out_token || !plan->host_token) return MQ_ERR_ARG;
    const MQStepPlan& q = *plan;
    if (q.weight_kind != 0 && q.weight_kind != 1) return MQ_ERR_ARG;
    if (q.row_pad_bytes != 0 && q.row_pad_bytes != ROW_SKEW) return MQ_ERR_ARG;
    if (input_token < 0 || input_token >= VOCAB) return MQ_ERR_TOKEN;
    int rc = check_common(q.embed_weight, q.layer_weights, q.final_norm_weight, q.lm_head_weight, q.cos_table,
                          q.sin_table, q.k_cache, q.v_cache, q.num_layers, position, q.max_seq_len);
    if (rc) return rc;
    if (q.weight_kind == 0 && (!q.lm_head_scale || !q.scales)) return MQ_ERR_ARG;
    DecodeParams P{};
    P.embed = q.embed_weight; P.layers = q.layer_weights; P.scales = q.scales; P.final_norm = q.final_norm_weight;
    P.lm_w = q.lm_head_weight; P.lm_scale = q.lm_head_scale;
    P.cos_t = (const __nv_bfloat16*)q.cos_table; P.sin_t = (const __nv_bfloat16*)q.sin_table;
    P.kc = (__nv_bfloat16*)q.k_cache; P.vc = (__nv_bfloat16*)q.v_cache;
    P.g_normalized = q.g_normalized;
    P.token_out = q.host_token;     // pinned host memory, written by the kernel's last CTA
    P.token_in = input_token; P.L = q.num_layers; P.position = position; P.max_seq = q.max_seq_len;
    P.attn_scale = q.attn_scale; P.row_pad = q.row_pad_bytes;
    *(volatile int*)q.host_token = -2;
    if ((rc = launch_step(q.weight_kind, P, stream))) return rc;
    cudaError_t e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return (int)e;
    const int t = *(volatile int*)q.host_token;
    if (t < 0) return MQ_ERR_DEVICE_STEP;
    *out_token = t;
    return 0;
}

extern "C" int mq_matvec(int weight_kind, const void* W, const float* scale, const float* x, float* y, int M, int K,
                         cudaStream_t stream) {
    if (!W || !x || !y || M <= 0) return MQ_ERR_ARG;
    if (weight_kind == 0 && !scale) return MQ_ERR_ARG;
    if (weight_kind != 0 && weight_kind != 1) return MQ_ERR_ARG;
    if (!aligned16(W) || !aligned16(x)) return MQ_ERR_ARG;
    if (K != 1024 && K != 2048 && K != 3072) return MQ_ERR_SIZE;
    DevState* d = nullptr;
    int rc = dev_state(&d);
    if (rc) return rc;
    MatvecParams P{W, scale, x, y, d->ws, g_budget_ns, M};
    void* args[] = {&P};
    const void* fn = nullptr;
#define MQ_MV_CASE(WT, KK)                                                                   \
    {                                                                                        \
        cudaError_t e = cudaFuncSetAttribute(matvec_kernel<WT, KK>,                          \
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                             (int)sizeof(Smem));                             \
        if (e != cudaSuccess) return (int)e;                                                 \
        fn = (const void*)matvec_kernel<WT, KK>;                                             \
    }
    if (weight_kind == 0) {
        if (K == 1024) MQ_MV_CASE(W8, 1024) else if (K == 2048) MQ_MV_CASE(W8, 2048) else MQ_MV_CASE(W8, 3072)
    } else {
        if (K == 1024) MQ_MV_CASE(W16, 1024) else if (K == 2048) MQ_MV_CASE(W16, 2048) else MQ_MV_CASE(W16, 3072)
    }
#undef MQ_MV_CASE
    return (int)cudaLaunchKernel(fn, dim3(d->num_sms), dim3(NTHREADS), args, sizeof(Smem), stream);
}

extern "C" int mq_device_status(int* code, int* info, int clear) {
    DevState* d = nullptr;
    int rc = dev_state(&d);
    if (rc) return rc;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return (int)e;
    int h[2] = {0, 0};
    e = cudaMemcpy(h, &d->ws->err_code, sizeof(h), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return (int)e;
    if (code) *code = h[0];
    if (info) *info = h[1];
    if (clear) {
        e = cudaMemset(&d->ws->err_code, 0, sizeof(h));
        if (e != cudaSuccess) return (int)e;
        e = cudaDeviceSynchronize();
    }
    return (int)e;
}

extern "C" int mq_set_wait_budget_ns(uint64_t ns) {
    if (ns == 0) return MQ_ERR_ARG;
    g_budget_ns = ns;
    return 0;
}

extern "C" int mq_inject_skip_publish(int enable, int cta) {
    g_skip_cta = enable ? cta : -1;
    return 0;
}

extern "C" int mq_kernel_info(int* num_ctas, int* smem_bytes, int* threads) {
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (num_ctas) *num_ctas = e == cudaSuccess ? sms : 0;
    if (smem_bytes) *smem_bytes = (int)sizeof(Smem);
    if (threads) *threads = NTHREADS;
    return (int)e;
}

extern "C" int mq_library_info(int* binary_version, int* workspace_allocated) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= MAX_DEV) return MQ_ERR_DEVICE;
    cudaFuncAttributes a{};
    if ((e = cudaFuncGetAttributes(&a, decode_kernel<W8>)) != cudaSuccess) return (int)e;
    if (binary_version) *binary_version = a.binaryVersion;
    if (workspace_allocated) *workspace_allocated = g_dev[dev].ws != nullptr ? 1 : 0;
    return 0;
}

extern "C" int mq_set_trace(unsigned long long* dev_buf, int slots_per_cta) {
    if (dev_buf && slots_per_cta <= 0) return MQ_ERR_ARG;
    g_trace = dev_buf;
    g_trace_slots = dev_buf ? slots_per_cta : 0;
    return 0;
}

// ===========================================================================
// Allocation-free INT8 decode step.
//
// Some callers cannot call cudaMalloc at the point where they decode: a plugin
// running inside a host framework that owns all device memory through its own
// pre-sized arena, a process whose allocator is locked after start-up, or code
// that must not allocate between the set-up and the serving loop.  For them the
// hand-off workspace of the decode kernel lives in the static device array
// below instead of in the lazily cudaMalloc'd one.  Every GPU that loads this
// library keeps these bytes resident until the process exits.
//
// Limit: the array holds exactly one Workspace (sizeof(mq::Workspace), about
// 0.8 MB), which serves models of up to MAX_LAYERS (32) layers and up to
// MAX_SPLITS (18) attention splits per KV head; num_layers above the limit is
// rejected with MQ_ERR_SIZE.
// ===========================================================================
static __device__ __align__(256) unsigned char g_static_workspace[sizeof(mq::Workspace)];

namespace {
struct StaticDevState {
    mq::Workspace* ws = nullptr;   // device address of g_static_workspace on this device
    int num_sms = 0;
    bool attr_set = false;
    unsigned long long epoch_used = 0;   // sum of the epoch increments of the launches since the last clear
};
StaticDevState g_static_dev[mq::MAX_DEV_STATIC];
}  // namespace

extern "C" int launch_a10_int8_decode_static(
    int input_token_id, int* output_token_id, const void* embed_weight, const LayerWeights* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight, const float* lm_head_scale, const void* cos_table,
    const void* sin_table, void* k_cache, void* v_cache, void* g_normalized, int num_layers, int position,
    int cache_len, int max_seq_len, float attn_scale, const ScalePointers* scales, cudaStream_t stream) {
    int rc = check_common(embed_weight, layer_weights, final_norm_weight, lm_head_weight, cos_table, sin_table,
                          k_cache, v_cache, num_layers, position, max_seq_len);
    if (rc) return rc;
    if (!output_token_id || !lm_head_scale || !scales) return MQ_ERR_ARG;
    if (cache_len != position + 1) return MQ_ERR_POSITION;
    if (input_token_id < 0 || input_token_id >= VOCAB) return MQ_ERR_TOKEN;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= MAX_DEV_STATIC) return MQ_ERR_DEVICE;
    StaticDevState& d = g_static_dev[dev];
    if (!d.ws) {
        // One-time set-up on this device (the device is current here): look up
        // the device address of the static array.  The name itself is only a
        // host-side stand-in and must never be handed to a kernel.
        void* ptr = nullptr;
        if ((e = cudaGetSymbolAddress(&ptr, g_static_workspace)) != cudaSuccess) return (int)e;
        int sms = 0;
        if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return (int)e;
        if (sms < MIN_CTAS) return MQ_ERR_DEVICE;
        d.ws = reinterpret_cast<Workspace*>(ptr);
        d.num_sms = sms;
    }
    if (!d.attr_set) {
        if ((e = cudaFuncSetAttribute(decode_kernel<W8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)sizeof(Smem))) != cudaSuccess)
            return (int)e;
        d.attr_set = true;
    }
    // The array keeps the previous call's contents.  Tags, counters and the
    // argmax slot are self-resetting; the error word must start at zero, and
    // the tagged buffers are cleared before their 32-bit epochs could wrap.
    const unsigned long long per_launch = (unsigned long long)(num_layers + 1) * TAGS_PER_LAYER;
    if (d.epoch_used + per_launch > 0xF0000000ull) {
        if ((e = cudaMemsetAsync(d.ws, 0, sizeof(Workspace), stream)) != cudaSuccess) return (int)e;
        d.epoch_used = 0;
    }
    if ((e = cudaMemsetAsync(&d.ws->err_code, 0, 2 * sizeof(int), stream)) != cudaSuccess) return (int)e;
    d.epoch_used += per_launch;
    DecodeParams P{};
    P.embed = embed_weight; P.layers = layer_weights; P.scales = scales; P.final_norm = final_norm_weight;
    P.lm_w = lm_head_weight; P.lm_scale = lm_head_scale;
    P.cos_t = (const __nv_bfloat16*)cos_table; P.sin_t = (const __nv_bfloat16*)sin_table;
    P.kc = (__nv_bfloat16*)k_cache; P.vc = (__nv_bfloat16*)v_cache;
    P.g_normalized = (float*)g_normalized; P.token_out = output_token_id;
    P.token_in = input_token_id; P.L = num_layers; P.position = position; P.max_seq = max_seq_len;
    P.attn_scale = attn_scale;
    P.ws = d.ws;
    P.budget_ns = g_budget_ns;
    P.skip_cta = g_skip_cta;   // test hook (mq_inject_skip_publish), one call only
    g_skip_cta = -1;
    P.splits = choose_splits(position + 1, d.num_sms);
    void* args[] = {&P};
    return (int)cudaLaunchCooperativeKernel((const void*)decode_kernel<W8>, dim3(d.num_sms), dim3(NTHREADS), args,
                                            sizeof(Smem), stream);
}
