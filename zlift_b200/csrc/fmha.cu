// fmha.cu -- fused flash-attention forward on the sm_100a tensor cores.
//
// Replaces the reference's fmha_run (zblas/zblas_gpu.cpp:892-1039): tiled
// online softmax over key tiles, causal mask `key > query + diag` with
// causal tile skipping (:932-934), P rounded to the input type before P.V,
// O accumulated in fp32 and normalised once at the end.  Adds the fp32
// log-sum-exp output the reference never writes.
//
// One CTA owns two 128-query tiles of one (batch, head) and walks the key
// tiles (128 keys) they need.  Ten warps:
//   warps 0-3   softmax for query tile 0, warps 4-7 for query tile 1:
//               tcgen05.ld a row of S = Q.K^T from TMEM (one thread per
//               query row), row max, exp2, row sum, write P (16-bit) back
//               into the same TMEM columns, rescale O in TMEM when the
//               running max grew by more than 2^8 (lazy rescaling: the
//               final O / l uses the same stale max, so the result is
//               exact), and at the end normalise O and store it with LSE.
//   warp 8      TMA producer: Q tiles once, then K_0, V_0, K_1, V_1, ...
//               through a ring of NSLOT tile slots, each released by the
//               MMA issuer as soon as its last reader has run (K_j after
//               the second tile's Q.K_j^T, V_j after its P.V_j), so loads
//               run well over a key step ahead.
//   warp 9      MMA issuer (one thread): S_t = Q_t.K_j^T (both operands in
//               shared memory) and O_t += P_t.V_j (P from TMEM, V in shared
//               memory), alternating the two query tiles so that one
//               tile's softmax overlaps the other tile's matrix products.
// TMEM columns: S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D, 256+2D).
#include "fmha.h"
#include "gemm.h"
#include "ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>

namespace zl {

namespace {

constexpr int BQ = 128;          // queries per tile
constexpr int BKEY = 128;        // keys per tile
constexpr int kThreads = 320;
constexpr float kLazyLog2 = 8.0f;   // rescale O only when the max grows by > 2^8

template <int D>
struct FCfg {
    static constexpr int BOXES = D / 64;                 // 128-byte column boxes per row
    static constexpr int TILE_BYTES = 128 * D * 2;       // one Q, K or V tile
    static constexpr int Q_OFF = 0;                      // two Q tiles
    static constexpr int KV_OFF = 2 * TILE_BYTES;        // K/V ring: slot s at +s*TILE
    static constexpr int SLOTS_FIT = (227 * 1024 - 1280 - KV_OFF) / TILE_BYTES;
    static constexpr int NSLOT = SLOTS_FIT > 8 ? 8 : SLOTS_FIT;
    static constexpr int BAR_OFF = KV_OFF + NSLOT * TILE_BYTES;
    static constexpr int SMEM = BAR_OFF + 256 + 1024;
    static_assert(NSLOT >= 4, "K/V ring too shallow");
    static_assert(SMEM <= 227 * 1024, "shared memory");
    static constexpr uint32_t S_COL0 = 0, S_COL1 = 128;
    static constexpr uint32_t O_COL0 = 256, O_COL1 = 256 + D;
    static constexpr uint32_t TMEM_COLS = 512;
};

struct FParams {
    int heads, kv_ratio, sq, sk;
    int npairs, nkt;             // query-tile pairs, key tiles
    int chunk;                   // (batch, head) pairs per scheduling chunk
    long long bh_begin, bh_count;
    long long ob, oh, orr;       // output strides (elements)
    void* o;
    float* lse;
    float scale, scale_log2;
    int causal, diag;
    int half_p;                  // P.V starts on the first half of P (see the MMA issuer)
    const uint16_t* bias;        // BIAS kernels: [b*bb + h*bh + query*br + key]
    long long bb, bh, br;
    int bias_vec;                // rows start 16-byte aligned: vector loads
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if constexpr (BF16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    } else {
        __half2 v = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
}

// number of key tiles query tile [q0, q0+128) needs
__device__ __forceinline__ int key_tiles(const FParams& p, int q0) {
    if (q0 >= p.sq) return 0;
    if (!p.causal) return p.nkt;
    const int last_q = min(q0 + BQ - 1, p.sq - 1);
    const int last_key = last_q + p.diag;
    if (last_key < 0) return 0;
    return min(last_key / BKEY + 1, p.nkt);
}

// Adds an additive bias row (16-bit, this thread's query row, keys
// key0..key0+127) to the raw scores in log2 units: s = s * c + bias * log2(e).
// Keys at or past `nvalid` get no bias (the mask sets them to -inf).
template <bool BF16>
__device__ __forceinline__ void bias_row(float (&s)[BKEY], const uint16_t* row, int nvalid,
                                         float c, bool vec) {
    constexpr float kLog2e = 1.4426950408889634f;
    auto cvt = [](uint32_t h) {
        if constexpr (BF16) return __uint_as_float(h << 16);
        else return __half2float(__ushort_as_half((unsigned short)h));
    };
    if (vec && nvalid >= BKEY) {
#pragma unroll
        for (int g = 0; g < BKEY / 8; g++) {
            const uint4 w = __ldg(reinterpret_cast<const uint4*>(row) + g);
            const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int t = 0; t < 4; t++) {
                s[8 * g + 2 * t] = fmaf(s[8 * g + 2 * t], c, cvt(u[t] & 0xffffu) * kLog2e);
                s[8 * g + 2 * t + 1] = fmaf(s[8 * g + 2 * t + 1], c, cvt(u[t] >> 16) * kLog2e);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < BKEY; i++) {
            const float bv = i < nvalid ? cvt(__ldg(row + i)) : 0.f;
            s[i] = fmaf(s[i], c, bv * kLog2e);
        }
    }
}

// BIAS: an additive bias of the input type is read from global memory for
// every score (the xformers block's attn_bias, zblas/zblas_gpu.cpp:963-966);
// scores are then kept in log2 units with the bias added before the mask.
template <int D, bool BF16, bool BIAS>
__global__ void __launch_bounds__(kThreads, 1)
fmha_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV,
                const FParams p) {
    using C = FCfg<D>;
    constexpr uint32_t IDESC_QK = make_idesc(1, BF16 ? 1 : 0, 0, 0, BQ, BKEY);
    constexpr uint32_t IDESC_PV = make_idesc(1, BF16 ? 1 : 0, 0, 1, BQ, D);
    constexpr int BOX_BYTES = 128 * 128;                 // 128 rows x 128 bytes

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int NSLOT = C::NSLOT;
    // a step's K and V sit in the ring at most NSLOT/2 + 1 steps ahead of
    // the MMA issuer, so KV_BARS such barriers are reused only after the
    // issuer has waited on them
    constexpr int KV_BARS = NSLOT / 2 + 1;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    uint64_t* qfull = bars + 0;
    uint64_t* sfull = bars + 1;       // [2] per query tile
    uint64_t* ofinal = bars + 3;      // [2]
    uint64_t* kvfull = bars + 5;      // [KV_BARS] K_j and V_j both landed (step j % KV_BARS)
    uint64_t* kvempty = kvfull + KV_BARS;   // [NSLOT] ring slot released
    // softmax -> MMA hand-off counts per query tile (4 warps add 1 each per
    // key tile): first half of P stored, all of P stored
    uint32_t* phalf = reinterpret_cast<uint32_t*>(kvempty + NSLOT);   // [2]
    uint32_t* pready = phalf + 2;                                      // [2]
    uint32_t* tmem_slot = pready + 2;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Blocks go in chunks of p.chunk (batch, head) pairs whose K and V fit
    // in L2 together; inside a chunk the query-tile pairs go heaviest first
    // across all its heads (with a causal mask the late pairs have the most
    // key tiles), so the last blocks to start are the shortest ones.
    const long long per_chunk = (long long)p.chunk * p.npairs;
    const long long ck = blockIdx.x / per_chunk;
    const int in_chunk = (int)(blockIdx.x - ck * per_chunk);
    const long long ck_heads = min((long long)p.chunk, p.bh_count - ck * p.chunk);
    const int pair = p.npairs - 1 - (int)(in_chunk / ck_heads);
    const long long bh = p.bh_begin + ck * p.chunk + in_chunk % ck_heads;
    const int b = (int)(bh / p.heads), h = (int)(bh % p.heads);
    const int hk = h / p.kv_ratio;
    // (scalars, not arrays: the warps index them by tile and an indexed array
    // would live in local memory)
    const int q00 = pair * 2 * BQ, q01 = q00 + BQ;
    const int nt0 = key_tiles(p, q00), nt1 = key_tiles(p, q01);
    const int nmax = max(nt0, nt1);

    if (threadIdx.x == 0) {
        mbar_init(qfull, 1);
        for (int i = 0; i < KV_BARS; i++) mbar_init(&kvfull[i], 1);
        for (int i = 0; i < NSLOT; i++) mbar_init(&kvempty[i], 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(&sfull[i], 1);
            mbar_init(&ofinal[i], 1);
            phalf[i] = 0;
            pready[i] = 0;
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 9) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 8) {
        // ---------------- TMA producer ----------------
        if (lane == 0 && nmax > 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            mbar_expect_tx(qfull, 2 * C::TILE_BYTES);
            for (int t = 0; t < 2; t++)
                for (int x = 0; x < C::BOXES; x++)
                    tma_load_4d(smem + C::Q_OFF + t * C::TILE_BYTES + x * BOX_BYTES, &tmQ, qfull,
                                x * 64, t ? q01 : q00, h, b);
            // item i: K_{i/2} (even i) or V_{i/2} (odd i), in slot i % NSLOT
            const int items = 2 * nmax;
            bool ok = true;
            for (int i = 0; i < items; i++) {
                const int slot = i % NSLOT;
                if (!mbar_wait(&kvempty[slot], ((i / NSLOT) & 1) ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                uint8_t* dst = smem + C::KV_OFF + slot * C::TILE_BYTES;
                uint64_t* full = &kvfull[(i >> 1) % KV_BARS];
                if (!(i & 1)) mbar_expect_tx(full, 2 * C::TILE_BYTES);
                const CUtensorMap* tm = (i & 1) ? &tmV : &tmK;
                for (int x = 0; x < C::BOXES; x++)
                    tma_load_4d(dst + x * BOX_BYTES, tm, full, x * 64, (i >> 1) * BKEY, hk, b);
            }
            // drain: the releases of the last NSLOT items are tcgen05.commit
            // arrivals on this CTA's barriers; none may still be in flight
            // when the CTA exits
            for (int i = items > NSLOT ? items - NSLOT : 0; ok && i < items; i++)
                ok = mbar_wait(&kvempty[i % NSLOT], (i / NSLOT) & 1, abort_flag);
        }
    } else if (warp == 9) {
        // ---------------- MMA issuer ----------------
        if (lane == 0 && nmax > 0) {
            const uint32_t sq_base = smem_u32(smem + C::Q_OFF);
            const uint32_t scol[2] = {C::S_COL0, C::S_COL1};
            const uint32_t ocol[2] = {C::O_COL0, C::O_COL1};
            // ring slot of K_j (item 2j) and V_j (item 2j+1); barrier and
            // wait parity of step j's pair
            auto slot_of = [](int item) { return item % NSLOT; };
            auto kv_wait = [&](int j) {
                return mbar_wait(&kvfull[j % KV_BARS], (uint32_t)((j / KV_BARS) & 1), abort_flag);
            };
            auto slot_addr = [&](int item) {
                return smem_u32(smem + C::KV_OFF + slot_of(item) * C::TILE_BYTES);
            };
            // The issuing thread is held at each tcgen05.mma about as long as
            // the MMA runs (N = 128), so the work between two MMAs is kept to
            // constant adds: a descriptor's start-address field is addr >> 4
            // in its low 14 bits, and a K step's byte offset adds to it
            // without carrying out (shared addresses are below 256 KB).
            auto issue_qk = [&](int t, int j) {
                const uint64_t kd = sw128_desc(slot_addr(2 * j), 16, 1024);
                const uint64_t qd = sw128_desc(sq_base + t * C::TILE_BYTES, 16, 1024);
                const uint32_t s_tm = tmem_base + scol[t];
#pragma unroll
                for (int ks = 0; ks < D / 16; ks++) {
                    const uint64_t off = ((ks >> 2) * BOX_BYTES + (ks & 3) * 32) >> 4;
                    mma_f16_ss(s_tm, qd + off, kd + off, IDESC_QK, ks > 0 ? 1u : 0u);
                }
                mma_commit(&sfull[t]);
            };
            // half 0: keys 0-63 of the tile, half 1: keys 64-127
            auto issue_pv = [&](int t, int j, int half) {
                const uint64_t vd = sw128_desc(slot_addr(2 * j + 1), BOX_BYTES, 1024);
                const uint32_t o_tm = tmem_base + ocol[t], p_tm = tmem_base + scol[t];
#pragma unroll
                for (int ks = half * (BKEY / 32); ks < (half + 1) * (BKEY / 32); ks++) {
                    // P: 16 keys = 8 packed TMEM columns per step; V: 16 key rows
                    mma_f16_ts(o_tm, p_tm + ks * 8, vd + ((ks * 16 * 128) >> 4), IDESC_PV,
                               (j > 0 || ks > 0) ? 1u : 0u);
                }
            };
            // Each ring item is released by one commit after its last reader:
            // tile 1 when it needs that key tile, else tile 0 (tile 1 has no
            // key tiles when its queries start past sq).  The ofinal commits
            // come after every release, so a CTA whose softmax warps have
            // seen both ofinal has no commit arrival left in flight but the
            // ones the producer drains.
            bool ok = mbar_wait(qfull, 0, abort_flag) && kv_wait(0);
            if (ok) {
                tc_fence_after();
                if (nt0 > 0) issue_qk(0, 0);
                if (nt1 > 0) issue_qk(1, 0);
                mma_commit(&kvempty[slot_of(0)]);
            }
            for (int j = 0; ok && j < nmax; j++) {
                bool have_next_k = false;
#pragma unroll
                for (int t = 0; t < 2; t++) {
                    const int ntt = t ? nt1 : nt0;
                    if (j >= ntt) continue;
                    const bool last_reader = t == 1 || j >= nt1;
                    // P.V on the first half of P while the softmax finishes the
                    // second (or on all of P at once: one wait fewer)
                    if (p.half_p) {
                        if (!flag_wait(&phalf[t], 4u * (j + 1), abort_flag)) { ok = false; break; }
                        tc_fence_after();
                        issue_pv(t, j, 0);
                    }
                    if (!flag_wait(&pready[t], 4u * (j + 1), abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    if (!p.half_p) issue_pv(t, j, 0);
                    issue_pv(t, j, 1);
                    if (last_reader) mma_commit(&kvempty[slot_of(2 * j + 1)]);
                    if (j + 1 == ntt) mma_commit(&ofinal[t]);
                    if (j + 1 < ntt) {
                        if (!have_next_k) {
                            if (!kv_wait(j + 1)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            have_next_k = true;
                        }
                        issue_qk(t, j + 1);
                        if (t == 1 || j + 1 >= nt1) mma_commit(&kvempty[slot_of(2 * j + 2)]);
                    }
                }
            }
        }
    } else {
        // ---------------- softmax + epilogue (warps 0-7) ----------------
        const int t = warp >> 2;
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const int tq0 = t ? q01 : q00;        // first query row of this tile
        const int tnt = t ? nt1 : nt0;        // key tiles this tile needs
        const int qrow = tq0 + r;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        const uint32_t s_addr = tmem_base + lane_off + (t ? C::S_COL1 : C::S_COL0);
        const uint32_t o_addr = tmem_base + lane_off + (t ? C::O_COL1 : C::O_COL0);
        // with a bias the scores are turned into log2 units (biased) right
        // after the load, and the rest of the softmax works with c = 1
        const float c = BIAS ? 1.f : p.scale_log2;
        const uint16_t* brow = nullptr;
        if constexpr (BIAS)
            brow = p.bias + (long long)b * p.bb + (long long)h * p.bh +
                   (long long)min(qrow, p.sq - 1) * p.br;
        float m_used = -INFINITY, l = 0.f;
        bool alive = true;
        for (int j = 0; j < tnt; j++) {
            if (!mbar_wait(&sfull[t], j & 1, abort_flag)) { alive = false; break; }
            tc_fence_after();
            float s[BKEY];
#pragma unroll
            for (int c0 = 0; c0 < BKEY; c0 += 32)
                tmem_ld32(s_addr + c0, *reinterpret_cast<uint32_t(*)[32]>(&s[c0]));
            tmem_wait_ld();
            const int key0 = j * BKEY;
            if constexpr (BIAS) bias_row<BF16>(s, brow + key0, p.sk - key0, p.scale_log2, p.bias_vec);
            const bool edge = (key0 + BKEY > p.sk) || (p.causal && key0 + BKEY - 1 > tq0 + p.diag);
            if (edge) {
                const int lim = p.causal ? min(p.sk - 1, qrow + p.diag) : p.sk - 1;
#pragma unroll
                for (int i = 0; i < BKEY; i++)
                    if (key0 + i > lim) s[i] = -INFINITY;
            }
            // row max over 8 independent partial maxima (short dependency chains)
            float mx8[8];
#pragma unroll
            for (int i = 0; i < 8; i++) mx8[i] = s[i];
#pragma unroll
            for (int i = 8; i < BKEY; i++) mx8[i & 7] = fmaxf(mx8[i & 7], s[i]);
            const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                   fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
            const float m_new = fmaxf(m_used, mx);
            if (j == 0) {
                m_used = m_new;
            } else {
                const bool resc = m_new != -INFINITY &&
                                  (m_used == -INFINITY || (m_new - m_used) * c > kLazyLog2);
                if (__any_sync(0xffffffffu, resc)) {
                    const float alpha = resc ? ex2((m_used - m_new) * c) : 1.f;
                    if (resc) {
                        l *= alpha;
                        m_used = m_new;
                    }
#pragma unroll 1
                    for (int c0 = 0; c0 < D; c0 += 16) {
                        uint32_t o[16];
                        tmem_ld16(o_addr + c0, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; i++)
                            o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st16(o_addr + c0, o);
                    }
                }
            }
            const float mc = m_used == -INFINITY ? 0.f : m_used * c;
            // exponentials on MUFU; row sum over 8 partial sums
            float sum8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            uint32_t pk[BKEY / 2];
            // two halves of the keys: P of keys 0-63 is stored and announced
            // (phalf) before the exponentials of keys 64-127, so P.V starts
            // while this warp is still working
#pragma unroll
            for (int half = 0; half < 2; half++) {
#pragma unroll
                for (int i = half * (BKEY / 4); i < (half + 1) * (BKEY / 4); i++) {
                    const float x0 = fmaf(s[2 * i], c, -mc), x1 = fmaf(s[2 * i + 1], c, -mc);
                    const float p0 = ex2(x0), p1 = ex2(x1);
                    sum8[i & 7] += p0 + p1;
                    pk[i] = pack2<BF16>(p0, p1);
                }
#pragma unroll
                for (int c0 = half * (BKEY / 4); c0 < (half + 1) * (BKEY / 4); c0 += 16)
                    tmem_st16(s_addr + c0, *reinterpret_cast<uint32_t(*)[16]>(&pk[c0]));
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) flag_add_release(half ? &pready[t] : &phalf[t]);
            }
            l += ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) +
                 ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
        }
        // ---- epilogue: O / l -> 16-bit, LSE ----
        bool have_o = tnt > 0 && alive;
        if (have_o) {
            if (!mbar_wait(&ofinal[t], 0, abort_flag)) have_o = false;
            else tc_fence_after();
        }
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const bool row_ok = qrow < p.sq;
        typedef uint16_t u16;
        u16* orow = static_cast<u16*>(p.o) + (long long)b * p.ob + (long long)h * p.oh +
                    (long long)qrow * p.orr;
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
            uint32_t v[32];
            if (have_o) {
                tmem_ld32(o_addr + c0, v);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) v[i] = 0u;
            }
            if (row_ok) {
                uint32_t w[16];
#pragma unroll
                for (int i = 0; i < 16; i++)
                    w[i] = pack2<BF16>(__uint_as_float(v[2 * i]) * inv,
                                       __uint_as_float(v[2 * i + 1]) * inv);
                uint4* dst = reinterpret_cast<uint4*>(orow + c0);
#pragma unroll
                for (int i = 0; i < 4; i++)
                    dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
            }
        }
        if (row_ok && p.lse) {
            // (m_used is in raw-score units, or in log2 units with a bias)
            const float lse_scale = BIAS ? 0.6931471805599453f : p.scale;
            const float lse = l > 0.f ? m_used * lse_scale + logf(l) : -INFINITY;
            p.lse[bh * (long long)p.sq + qrow] = lse;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
    static std::atomic<EncodeFn> fn{nullptr};
    EncodeFn f = fn.load();
    if (f) return f;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess) {
        f = reinterpret_cast<EncodeFn>(ptr);
        fn.store(f);
    }
    return f;
}

// [batch][seq][heads][d] view of one operand: dims {d, seq, heads, batch}
bool attn_tmap(CUtensorMap* tm, int elem, const void* base, int d, int seq, int heads,
               int batch, long long rs, long long hs, long long bs) {
    EncodeFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)seq, (cuuint64_t)heads, (cuuint64_t)batch};
    auto fix = [](long long s) { return (cuuint64_t)(s * 2 > 0 ? s * 2 : 16); };
    cuuint64_t strides[3] = {fix(rs), fix(hs), fix(bs)};
    cuuint32_t box[4] = {64, 128, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(tm, elem == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                     4, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int D, bool BF16, bool BIAS>
int launch(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v, const FParams& p,
           long long grid, cudaStream_t s) {
    using C = FCfg<D>;
    auto kern = fmha_fwd_kernel<D, BF16, BIAS>;
    static std::atomic<unsigned long long> attr_set{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return (int)e;
        attr_set.fetch_or(bit);
    }
    kern<<<(unsigned)grid, kThreads, C::SMEM, s>>>(q, k, v, p);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e == cudaSuccess ? 0 : (int)e;
}

template <int D, bool BF16>
int launch_bias(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                const FParams& p, long long grid, cudaStream_t s) {
    return p.bias ? launch<D, BF16, true>(q, k, v, p, grid, s)
                  : launch<D, BF16, false>(q, k, v, p, grid, s);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int fmha_fwd(const AttnDesc& d, cudaStream_t s) {
    if (d.elem == 2) return attn_f32_fwd(d, s);
    if (d.elem != 0 && d.elem != 1) return 1;
    if (d.d != 64 && d.d != 128) return 1;
    if (d.batches <= 0 || d.heads <= 0 || d.sq <= 0 || d.sk <= 0 || d.kv_ratio <= 0) return 1;
    if (d.heads % d.kv_ratio) return 1;
    if (!al16(d.q) || !al16(d.k) || !al16(d.v) || !al16(d.o)) return 1;
    // TMA strides: multiples of 16 bytes; output rows written as 16-byte vectors
    for (long long st : {d.qr, d.qh, d.qb, d.kr, d.kh, d.kb, d.vr, d.vh, d.vb})
        if ((st * 2) % 16) return 1;
    if ((d.orr * 2) % 16 || (d.oh * 2) % 16 || (d.ob * 2) % 16) return 1;
    if (d.qr <= 0 || d.kr <= 0 || d.vr <= 0) return 1;
    const int hk = d.heads / d.kv_ratio;
    CUtensorMap tq, tk, tv;
    if (!attn_tmap(&tq, d.elem, d.q, d.d, d.sq, d.heads, d.batches, d.qr, d.qh, d.qb)) return 1;
    if (!attn_tmap(&tk, d.elem, d.k, d.d, d.sk, hk, d.batches, d.kr, d.kh, d.kb)) return 1;
    if (!attn_tmap(&tv, d.elem, d.v, d.d, d.sk, hk, d.batches, d.vr, d.vh, d.vb)) return 1;
    FParams p;
    p.heads = d.heads;
    p.kv_ratio = d.kv_ratio;
    p.sq = d.sq;
    p.sk = d.sk;
    p.npairs = (d.sq + 2 * BQ - 1) / (2 * BQ);
    p.nkt = (d.sk + BKEY - 1) / BKEY;
    const long long total_bh = (long long)d.batches * d.heads;
    p.bh_begin = d.pair_end > 0 ? d.pair_begin : 0;
    p.bh_count = d.pair_end > 0 ? d.pair_end - d.pair_begin : total_bh;
    if (p.bh_count <= 0) return 0;
    p.ob = d.ob; p.oh = d.oh; p.orr = d.orr;
    p.o = d.o;
    p.lse = d.lse;
    p.scale = d.scale;
    p.scale_log2 = d.scale * 1.4426950408889634f;
    p.causal = d.causal ? 1 : 0;
    p.diag = d.diag;
    // P.V on all of P at once (one wait per tile and key tile) measured 2-6 %
    // faster than starting on its first half; ZBLAS_FMHA_HALF=1 restores that
    p.half_p = getenv("ZBLAS_FMHA_HALF") ? 1 : 0;
    p.bias = static_cast<const uint16_t*>(d.bias);
    p.bb = d.bb; p.bh = d.bh; p.br = d.br;
    p.bias_vec = d.bias && al16(d.bias) && (d.br * 2) % 16 == 0 && (d.bh * 2) % 16 == 0 &&
                 (d.bb * 2) % 16 == 0;
    const long long grid = (long long)p.npairs * p.bh_count;
    if (grid > 0x7fffffffLL) return 1;
    // scheduling chunks: the (batch, head) pairs whose K and V fit in 16 MB,
    // rounded down to a power of two (8 heads of 4096 keys at head_dim 128).
    // Measured on B200 with the causal 4096-key case over 256 and over 32
    // heads: chunks of 8 ran 2.6 % and 20 % faster than head-by-head order;
    // 8-32 were within 1 % of each other, chunks that split the heads
    // unevenly (12, 24) or small ones (2, 4) slower.  ZBLAS_FMHA_CHUNK
    // overrides (1 = head by head).
    {
        const long long kv = 2LL * d.sk * d.d * 2;
        const long long fit = kv > 0 ? std::max(1LL, (16LL << 20) / kv) : 1;
        long long ch = 1;
        while (ch * 2 <= fit) ch *= 2;
        if (const char* e = getenv("ZBLAS_FMHA_CHUNK")) ch = atoll(e);
        p.chunk = (int)std::max(1LL, std::min(ch, p.bh_count));
    }
    if (d.d == 128)
        return d.elem == 1 ? launch_bias<128, true>(tq, tk, tv, p, grid, s)
                           : launch_bias<128, false>(tq, tk, tv, p, grid, s);
    return d.elem == 1 ? launch_bias<64, true>(tq, tk, tv, p, grid, s)
                       : launch_bias<64, false>(tq, tk, tv, p, grid, s);
}

int fmha_set_wait_limit(unsigned long long ns) { return set_unit_wait_limit(ns); }

int fmha_error(bool clear) {
    int v = 0;
    cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(int));
    if (clear && v) {
        int z = 0;
        cudaMemcpyToSymbol(g_dev_error, &z, sizeof(int));
    }
    return v;
}

}  // namespace zl
