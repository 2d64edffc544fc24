// gemm_tc.cu -- column-major GEMM on the sm_100a tensor cores.
//
// Replaces the reference's XMX GEMMs (zblas/zblas_gpu.cpp: mad_h :405-497
// for 16-bit inputs, mad :266-332 with split_to_bf16 :219-265 for fp32) and
// adds the int8 x int8 -> int32 path the reference lacks.
//
// One persistent CTA per SM walks output tiles of 128 x BN (rows of C x
// columns of C).  Six warps, each with one job:
//   warp 0      TMA producer: loads 128-byte-swizzled A and B tiles into a
//               STAGES-deep shared-memory ring (full/empty mbarriers).
//   warp 1      MMA issuer: allocates TMEM, issues tcgen05.mma from one
//               thread into one of two TMEM accumulators, and commits each
//               stage back to the producer and each finished tile to the
//               epilogue.
//   warps 2-5   epilogue: tcgen05.ld the accumulator (warp w reads TMEM
//               lanes 32*(w%4)..+31, i.e. rows of the tile), apply
//               alpha*acc + beta*C, convert, store to C.  The two TMEM
//               accumulators let the epilogue of tile i overlap the main
//               loop of tile i+1.
// When the last wave of tiles would leave more than half of the CTAs idle,
// each of its tiles is split along K into 2-4 parts run by different CTAs
// (see unit_of and last_part): the parts park their partial sums in a
// workspace, and the part that finishes last adds them up in part order and
// runs the epilogue.
// Column-major operands need no staging transpose (the reference's
// stage_tight, zblas_gpu.cpp:633-669): an operand whose contiguous
// dimension is M or N is described to the tensor core as "MN-major".
#include "gemm.h"
#include "ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <string>

namespace zl {

namespace {

constexpr int BM = 128;
constexpr int kThreads = 192;
constexpr int kSmemBudget = 227 * 1024;     // dynamic shared memory per CTA
constexpr int kSmemReserve = 1024 + 256;    // alignment slack + barriers

template <int KIND> struct KT;
template <> struct KT<(int)Kind::F16>    { static constexpr int es = 2, uk = 16, cfmt = 1, abfmt = 0, planes = 1; };
template <> struct KT<(int)Kind::BF16>   { static constexpr int es = 2, uk = 16, cfmt = 1, abfmt = 1, planes = 1; };
template <> struct KT<(int)Kind::TF32X3> { static constexpr int es = 4, uk = 8,  cfmt = 1, abfmt = 2, planes = 2; };
template <> struct KT<(int)Kind::TF32>   { static constexpr int es = 4, uk = 8,  cfmt = 1, abfmt = 2, planes = 1; };
template <> struct KT<(int)Kind::I8>     { static constexpr int es = 1, uk = 32, cfmt = 2, abfmt = 1, planes = 1; };

// bytes of one output element
__host__ __device__ constexpr int out_es(int out) {
    return out == kR8I ? 1 : (out == kR16F || out == kR16BF) ? 2 : 4;
}
// outputs computed from an int32 accumulator (int32 C, or int8 C requantised)
__host__ __device__ constexpr bool int_acc(int out) { return out == kR32I || out == kR8I; }

struct TcParams {
    int m, n, k, batch;
    int tiles_m, tiles_n, k_blocks;
    long long ldc, strideC;
    void* C;
    int out_type;
    float alpha, beta;
    int32_t ialpha, ibeta;
    const void* alpha_dev;
    const void* beta_dev;
    int epi;                 // EpiFlags (floating-point outputs)
    const void* bias;
    int bias_type;
    // Units of work: units [0, main_units) are whole tiles (unit u = tile
    // u); each later tile is split along K into `split` units.  split == 1:
    // main_units = total_units = number of tiles.
    int main_units, total_units, split;
    // tail_halves: the tiles after main_units are each two units of BN/2
    // columns (an N split of a sparse last wave) instead of K-split parts
    int tail_halves;
    int kc;                          // K blocks per accumulation chunk (see fold_chunks)
    uint32_t* work;                  // partial sums of split tiles (fp32 or int32 bits)
    size_t work_bytes;
    unsigned long long* counters;    // per (split tile, CTA rank): epoch << 16 | parts done
    unsigned long long epoch;        // this launch's tag, < 2^48
};

// What one unit of work covers: output tile `t` and K blocks [kb0, kb1);
// part >= 0 for a K-split unit; nh = 1 or 2 for the first or second
// BN/2-column half of a tile (0: the whole tile).
struct Unit {
    int t, kb0, kb1, part, nh;
};

__device__ __forceinline__ Unit unit_of(const TcParams& p, int u) {
    Unit r;
    r.nh = 0;
    if (u < p.main_units) {
        r.t = u;
        r.kb0 = 0;
        r.kb1 = p.k_blocks;
        r.part = -1;
    } else if (p.tail_halves) {
        const int v = u - p.main_units;
        r.t = p.main_units + v / 2;
        r.kb0 = 0;
        r.kb1 = p.k_blocks;
        r.part = -1;
        r.nh = 1 + (v & 1);
    } else {
        const int v = u - p.main_units;
        const int s = v % p.split;
        r.t = p.main_units + v / p.split;
        r.part = s;
        r.kb0 = (int)((long long)s * p.k_blocks / p.split);
        r.kb1 = (int)((long long)(s + 1) * p.k_blocks / p.split);
    }
    return r;
}

// Counts one finished part of split tile `tt` (this CTA's rows); true for
// the part that completes the tile.  The counter carries the launch's epoch
// so a count left by an aborted launch reads as zero; the last part resets
// it, so a CUDA graph replaying this launch with the same epoch starts from
// zero too.  No CTA ever waits for another.
__device__ __forceinline__ bool last_part(unsigned long long* counters, unsigned long long epoch,
                                          int split, int slot) {
    unsigned long long* c = counters + slot;
    unsigned long long cur = atomicAdd(c, 0ull);
    while (true) {
        const unsigned long long done = (cur >> 16) == epoch ? (cur & 0xffffull) : 0ull;
        const unsigned long long next = (epoch << 16) | (done + 1);
        const unsigned long long prev = atomicCAS(c, cur, next);
        if (prev == cur) {
            if (done + 1 < (unsigned long long)split) return false;
            atomicExch(c, 0ull);
            return true;
        }
        cur = prev;
    }
}

// Sum over the parts of a split tile (2 to 4), in part order, for this
// thread's row and 32 columns: part `own` is v (this CTA's accumulator);
// the others come from `staged`, their 32 x 128 chunks one after another
// in part order with `own` left out.  Part order makes the bits independent
// of which part completed the tile.  16 columns at a time, parts in a loop,
// a part's 16 loads unrolled so they are in flight together.
template <int OUT>
__device__ __forceinline__ void combine_parts(uint32_t (&v)[32], const uint32_t* staged,
                                              int split, int own, int row) {
#pragma unroll
    for (int h = 0; h < 2; h++) {
        uint32_t acc[16];
        const uint32_t* src = staged + row + h * 16 * BM;
        for (int q = 0; q < split; q++) {
            uint32_t x[16];
            if (q == own) {
#pragma unroll
                for (int j = 0; j < 16; j++) x[j] = v[h * 16 + j];
            } else {
#pragma unroll
                for (int j = 0; j < 16; j++) x[j] = src[j * BM];
                src += 32 * BM;
            }
#pragma unroll
            for (int j = 0; j < 16; j++) {
                if constexpr (int_acc(OUT)) acc[j] = q ? acc[j] + x[j] : x[j];
                else acc[j] = q ? __float_as_uint(__uint_as_float(acc[j]) + __uint_as_float(x[j])) : x[j];
            }
        }
#pragma unroll
        for (int j = 0; j < 16; j++) v[h * 16 + j] = acc[j];
    }
}

// Chunked accumulation (the 3xTF32 kernel): the tensor core's fp32
// accumulation of tf32 products loses precision at every step, so the error
// of one long accumulation grows with K.  The MMA issuer starts a fresh
// accumulator every kc K blocks; the epilogue adds the chunks up in fp32
// registers, round to nearest, in K order: fold_chunk for every chunk but a
// unit's last, add_run into the last chunk's TMEM columns.
template <int BN>
__device__ __forceinline__ void fold_chunk(uint32_t taddr, float (&run)[BN], bool first) {
#pragma unroll
    for (int i = 0; i < BN / 32; i++) {
        uint32_t v[32];
        tmem_ld32(taddr + i * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; j++)
            run[i * 32 + j] = first ? __uint_as_float(v[j]) : run[i * 32 + j] + __uint_as_float(v[j]);
    }
}

template <int BN>
__device__ __forceinline__ void add_run(uint32_t taddr, const float (&run)[BN]) {
#pragma unroll
    for (int i = 0; i < BN / 32; i++) {
        uint32_t v[32];
        tmem_ld32(taddr + i * 32, v);
        tmem_wait_ld();
        uint32_t lo[16], hi[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            lo[j] = __float_as_uint(run[i * 32 + j] + __uint_as_float(v[j]));
            hi[j] = __float_as_uint(run[i * 32 + 16 + j] + __uint_as_float(v[16 + j]));
        }
        tmem_st16(taddr + i * 32, lo);
        tmem_st16(taddr + i * 32 + 16, hi);
    }
    tmem_wait_st();
}

// bias[row] as float (0 past the end or without a bias)
__device__ __forceinline__ float load_bias(const TcParams& p, long long row) {
    if (!(p.epi & kEpiBias) || !p.bias || row >= p.m) return 0.f;
    switch (p.bias_type) {
    case kR16F: return __half2float(static_cast<const __half*>(p.bias)[row]);
    case kR16BF: return __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[row]);
    default: return static_cast<const float*>(p.bias)[row];
    }
}


// Epilogue staging: two buffers of 32 output columns x 128 rows, laid out
// [column][row] (rows contiguous, as in column-major C), moved to and from
// global memory by TMA.  EPI_ES = 0: no staging (direct stores).
constexpr int kEpiCols = 32;

template <int BN, int KIND, int EPI_ES, bool PAIR = false>
struct Cfg {
    static constexpr int es = KT<KIND>::es;
    static constexpr int BK = 128 / es;          // K elements per stage (one 128-byte row)
    static constexpr int BOX = 128 / es;         // MN elements in one 128-byte row
    static constexpr int A_BYTES = BM * 128;
    // a CTA pair splits B's BN columns: each CTA holds BN/2 of them
    static constexpr int B_ROWS = PAIR ? BN / 2 : BN;
    static constexpr int B_BYTES = B_ROWS * 128;
    static constexpr int PLANES = KT<KIND>::planes;
    static constexpr int STAGE_BYTES = (A_BYTES + B_BYTES) * PLANES;
    static constexpr int EPI_BUF = kEpiCols * BM * EPI_ES;     // one staging buffer
    static constexpr int NEPI = 2;                              // staging buffers
    static constexpr int EPI_BYTES = NEPI * EPI_BUF;
    static constexpr int STAGES_FIT = (kSmemBudget - kSmemReserve - EPI_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
    static constexpr int TMEM_COLS = (2 * BN) < 32 ? 32 : (2 * BN);
    static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_BYTES + kSmemReserve;
    static_assert(STAGES >= 2, "shared memory too small for a two-stage ring");
};

// Tile index -> (batch, tile row, tile column), walking groups of 8 tile
// rows so that consecutive CTAs share B columns in L2 (the role of the
// reference's slab rasterisation, zblas_gpu.cpp:414-430 / :498-504).
__device__ __forceinline__ void decode_tile(int t, int tiles_m, int tiles_n,
                                            int& b, int& tm, int& tn) {
    const int per_b = tiles_m * tiles_n;
    b = t / per_b;
    const int r = t - b * per_b;
    constexpr int G = 8;
    const int group = r / (G * tiles_n);
    const int first = group * G;
    const int gm = min(tiles_m - first, G);
    const int rr = r - group * G * tiles_n;
    tm = first + rr % gm;
    tn = rr / gm;
}

// One operand tile (ROWS of M or N by BK of K) into shared memory.
//  K-major:  tensor map dims {K, MN, batch}, one box {BK, ROWS, 1}; row r
//            of the tile (128 bytes) lands at r*128, 16-byte chunks XORed
//            with r%8 (128-byte swizzle).
//  MN-major: tensor map dims {MN, K, batch}, ROWS/BOX boxes {BOX, BK, 1};
//            box i holds MN elements [i*BOX, (i+1)*BOX) for all BK values
//            of K, K row kk at kk*128 within the box.
template <bool MN, int ROWS, int BK, int BOX>
__device__ __forceinline__ void load_operand(uint8_t* dst, const CUtensorMap* tm,
                                             uint64_t* bar, int mn0, int k0, int b) {
    static_assert(!MN || ROWS % BOX == 0, "an MN-major tile is made of whole swizzle rows");
    if constexpr (!MN) {
        tma_load_3d(dst, tm, bar, k0, mn0, b);
    } else {
#pragma unroll
        for (int i = 0; i < ROWS / BOX; i++)
            tma_load_3d(dst + i * (BK * 128), tm, bar, mn0 + i * BOX, k0, b);
    }
}

// Pair form: completion bytes go to the leader CTA's barrier `bar0`
// (shared::cluster address).
template <bool MN, int ROWS, int BK, int BOX>
__device__ __forceinline__ void load_operand_pair(uint8_t* dst, const CUtensorMap* tm,
                                                  uint32_t bar0, int mn0, int k0, int b) {
    static_assert(!MN || ROWS % BOX == 0, "an MN-major tile is made of whole swizzle rows");
    if constexpr (!MN) {
        tma_load_3d_pair(dst, tm, bar0, k0, mn0, b);
    } else {
#pragma unroll
        for (int i = 0; i < ROWS / BOX; i++)
            tma_load_3d_pair(dst + i * (BK * 128), tm, bar0, mn0 + i * BOX, k0, b);
    }
}

// An epilogue warp is done with an accumulator: arrive on the MMA issuer's
// barrier (the leader CTA's, for a pair).
__device__ __forceinline__ void release_acc(uint64_t* bar, uint32_t rank) {
    if (rank == 0) mbar_arrive(bar);
    else mbar_arrive_cluster(mapa_shared(bar, 0));
}

// Descriptor of K step `ks` (uk elements of K) of an operand tile.
//  K-major:  8-row core groups 1024 bytes apart (SBO); the K step moves the
//            start address along the 128-byte row.
//  MN-major: 64/32/128-element MN blocks BK*128 bytes apart (LBO), 8-row K
//            groups 1024 bytes apart (SBO); the K step skips uk rows.
template <bool MN, int BK, int UK>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int ks) {
    if constexpr (!MN) {
        return sw128_desc(base + ks * 32, 16, 1024);
    } else {
        return sw128_desc(base + ks * UK * 128, BK * 128, 1024);
    }
}

// Raw bits of C's old value (for beta * C), read ahead of the stores.
template <int OUT>
__device__ __forceinline__ uint32_t load_c(const void* C, long long at) {
    if constexpr (OUT == kR8I)
        return static_cast<const uint8_t*>(C)[at];
    else if constexpr (OUT == kR16F || OUT == kR16BF)
        return static_cast<const uint16_t*>(C)[at];
    else
        return static_cast<const uint32_t*>(C)[at];
}

// alpha * acc + beta * old, converted to the output type and stored.
template <int OUT>
__device__ __forceinline__ void store_out(void* C, long long at, uint32_t raw, uint32_t old,
                                          bool use_beta, float alpha, float beta,
                                          int32_t ia, int32_t ib, int epi, float bias_row) {
    if constexpr (OUT == kR32I) {
        uint32_t v = (uint32_t)ia * raw;                 // two's-complement wrap
        if (use_beta) v += (uint32_t)ib * old;
        static_cast<int32_t*>(C)[at] = (int32_t)v;
    } else if constexpr (OUT == kR8I) {
        static_cast<int8_t*>(C)[at] =
            requant_s8((int32_t)raw, alpha, use_beta, beta, (int8_t)(uint8_t)old);
    } else {
        float v = alpha * __uint_as_float(raw);
        if constexpr (OUT == kR32F) {
            if (use_beta) v = fmaf(beta, __uint_as_float(old), v);
            if (epi) v = apply_act(v + bias_row, epi);
            static_cast<float*>(C)[at] = v;
        } else if constexpr (OUT == kR16F) {
            if (use_beta) v = fmaf(beta, __half2float(__ushort_as_half((unsigned short)old)), v);
            if (epi) v = apply_act(v + bias_row, epi);
            static_cast<__half*>(C)[at] = __float2half_rn(v);
        } else {
            if (use_beta)
                v = fmaf(beta, __bfloat162float(__ushort_as_bfloat16((unsigned short)old)), v);
            if (epi) v = apply_act(v + bias_row, epi);
            static_cast<__nv_bfloat16*>(C)[at] = __float2bfloat16_rn(v);
        }
    }
}

// alpha * acc (+ beta * C already in the staging buffer) (+ bias, act),
// converted in place: this thread's row of one 32-column staging chunk
// ([column][row], 128 rows).  BETA and ACT are compile-time so that each
// loop body holds only the arithmetic it runs: with run-time flags inside
// the unrolled loop the compiler predicated the activation (tanhf) for
// every element, which made this conversion cost ~1250 clocks per chunk.
template <int OUT, bool BETA, bool ACT>
__device__ __forceinline__ void convert_chunk_t(const uint32_t (&v)[32], uint8_t* sbuf, int row,
                                                float alpha, float beta, int32_t ia, int32_t ib,
                                                int epi, float bias_row) {
    constexpr int ES = out_es(OUT);
#pragma unroll
    for (int j = 0; j < 32; j++) {
        uint8_t* e = sbuf + (j * BM + row) * ES;
        if constexpr (OUT == kR32I) {
            uint32_t x = (uint32_t)ia * v[j];
            if constexpr (BETA) x += (uint32_t)ib * *reinterpret_cast<uint32_t*>(e);
            *reinterpret_cast<uint32_t*>(e) = x;
        } else if constexpr (OUT == kR8I) {
            *reinterpret_cast<int8_t*>(e) =
                requant_s8((int32_t)v[j], alpha, BETA, beta, BETA ? *reinterpret_cast<int8_t*>(e) : 0);
        } else {
            float x = alpha * __uint_as_float(v[j]);
            if constexpr (OUT == kR32F) {
                if constexpr (BETA) x = fmaf(beta, *reinterpret_cast<float*>(e), x);
                if constexpr (ACT) x = apply_act(x + bias_row, epi);
                *reinterpret_cast<float*>(e) = x;
            } else if constexpr (OUT == kR16F) {
                if constexpr (BETA) x = fmaf(beta, __half2float(*reinterpret_cast<__half*>(e)), x);
                if constexpr (ACT) x = apply_act(x + bias_row, epi);
                *reinterpret_cast<__half*>(e) = __float2half_rn(x);
            } else {
                if constexpr (BETA)
                    x = fmaf(beta, __bfloat162float(*reinterpret_cast<__nv_bfloat16*>(e)), x);
                if constexpr (ACT) x = apply_act(x + bias_row, epi);
                *reinterpret_cast<__nv_bfloat16*>(e) = __float2bfloat16_rn(x);
            }
        }
    }
}

template <int OUT>
__device__ __forceinline__ void convert_chunk(const uint32_t (&v)[32], uint8_t* sbuf, int row,
                                              float alpha, float beta, int32_t ia, int32_t ib,
                                              bool use_beta, int epi, float bias_row) {
    if constexpr (int_acc(OUT)) {
        if (use_beta) convert_chunk_t<OUT, true, false>(v, sbuf, row, alpha, beta, ia, ib, 0, 0.f);
        else convert_chunk_t<OUT, false, false>(v, sbuf, row, alpha, beta, ia, ib, 0, 0.f);
    } else if (epi) {
        if (use_beta) convert_chunk_t<OUT, true, true>(v, sbuf, row, alpha, beta, ia, ib, epi, bias_row);
        else convert_chunk_t<OUT, false, true>(v, sbuf, row, alpha, beta, ia, ib, epi, bias_row);
    } else {
        if (use_beta) convert_chunk_t<OUT, true, false>(v, sbuf, row, alpha, beta, ia, ib, 0, 0.f);
        else convert_chunk_t<OUT, false, false>(v, sbuf, row, alpha, beta, ia, ib, 0, 0.f);
    }
}

// What a K-split unit's epilogue needs (by value: the function below is
// out of line, and taking the address of the kernel's parameters would make
// the kernel copy them).
struct SplitArgs {
    uint32_t* work;
    unsigned long long* counters;
    unsigned long long epoch;
    int split, tt, part, rank, ncols;
    uint32_t taddr;
    int m0, n0, b;
    float alpha, beta, bias_row;
    int32_t ia, ib;
    int epi;
    bool use_beta;
};
struct EpiState {
    int chunk;
    uint32_t cphase, rphase;
    bool ok;
};

// Epilogue of a K-split unit, out of line so that the tile epilogue's hot
// loop is compiled as if splits did not exist (inlined, its code cost the
// 256 x 512^3 batched bf16 GEMM 35 %).  The part stores its partial sums
// ([column][row] of this CTA's 128 rows), counts itself, and goes on only
// if it completed the tile: then it copies the other parts' sums chunk by
// chunk (32 columns, 16 KB per part) into the operand ring, idle by now (a
// split unit is its CTA's last), up to three chunks ahead, adds them in part
// order and runs the staged epilogue on the result.  Every sync point is
// uniform over the 128 epilogue threads, as in the kernel.
template <int BN, int OUT, bool PAIR, int NEPI, int EPI_BUF, int RING_BYTES>
__device__ __noinline__ EpiState split_unit_epilogue(const SplitArgs a, EpiState st, uint8_t* smem,
                                                     uint8_t* epi, uint64_t* cbar, uint64_t* rbar,
                                                     volatile int* abort_flag,
                                                     volatile int* split_last,
                                                     const CUtensorMap* tmC, int row, int lane,
                                                     bool leader) {
    constexpr int RANKS = PAIR ? 2 : 1;
    constexpr uint32_t kChunkBytes = 32 * BM * 4;
    const size_t tile_words = (size_t)BN * BM;
    uint32_t* mine = a.work + (((size_t)a.tt * a.split + a.part) * RANKS + a.rank) * tile_words;
#pragma unroll 1
    for (int c0 = 0; c0 < a.ncols; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(a.taddr + c0, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; j++) __stcg(mine + (size_t)(c0 + j) * BM + row, v[j]);
    }
    // the partial sums are read by another CTA's bulk copies (async proxy)
    fence_async_global();
    __threadfence();
    named_bar_sync(1, 128);
    if (leader)
        *split_last = last_part(a.counters, a.epoch, a.split, a.tt * RANKS + a.rank) ? 1 : 0;
    named_bar_sync(1, 128);
    if (!*split_last) return st;
    __threadfence();
    // the other parts' plain stores, acquired through the counter, before
    // this CTA's bulk copies read them
    fence_async_global();
    const int own = a.part;
    const uint32_t* part0 = a.work + ((size_t)a.tt * a.split * RANKS + a.rank) * tile_words;
    const int rslots = max(1, min(3, RING_BYTES / ((a.split - 1) * (int)kChunkBytes)));
    auto fetch = [&](int c) {                  // leader: chunk c of the other parts
        const int sl = c % rslots;
        uint8_t* dst = smem + (size_t)sl * (a.split - 1) * kChunkBytes;
        mbar_expect_tx(&rbar[sl], (uint32_t)(a.split - 1) * kChunkBytes);
        for (int q = 0, i = 0; q < a.split; q++) {
            if (q == own) continue;
            bulk_load(dst + (size_t)i * kChunkBytes,
                      part0 + (size_t)q * RANKS * tile_words + (size_t)c * 32 * BM, kChunkBytes,
                      &rbar[sl]);
            i++;
        }
    };
    if (leader)
        for (int c = 0; c < rslots && c * 32 < a.ncols; c++) fetch(c);
#pragma unroll 1
    for (int c0 = 0; c0 < a.ncols; c0 += kEpiCols, st.chunk++) {
        const int buf = st.chunk % NEPI, nbuf = (st.chunk + 1) % NEPI;
        uint8_t* sbuf = epi + buf * EPI_BUF;
        if (leader) {
            if (a.use_beta) {
                if (c0 == 0) {
                    bulk_wait_read<NEPI - 1>();
                    mbar_expect_tx(&cbar[buf], EPI_BUF);
                    tma_load_3d(sbuf, tmC, &cbar[buf], a.m0, a.n0 + c0, a.b);
                }
                if (c0 + kEpiCols < a.ncols) {
                    bulk_wait_read<NEPI - 2>();
                    mbar_expect_tx(&cbar[nbuf], EPI_BUF);
                    tma_load_3d(epi + nbuf * EPI_BUF, tmC, &cbar[nbuf], a.m0,
                                a.n0 + c0 + kEpiCols, a.b);
                }
            } else {
                bulk_wait_read<NEPI - 1>();
            }
        }
        uint32_t v[32];
        tmem_ld32(a.taddr + c0, v);
        bool w = true;
        if (a.use_beta) {
            w = mbar_wait(&cbar[buf], (st.cphase >> buf) & 1u, abort_flag);
            st.cphase ^= 1u << buf;
        }
        const int sl = (c0 / 32) % rslots;
        w = mbar_wait(&rbar[sl], (st.rphase >> sl) & 1u, abort_flag) && w;
        st.rphase ^= 1u << sl;
        tmem_wait_ld();
        st.ok = named_bar_and(1, 128, w);
        if (!st.ok) return st;
        combine_parts<OUT>(v,
                           reinterpret_cast<const uint32_t*>(smem + (size_t)sl * (a.split - 1) *
                                                                        kChunkBytes),
                           a.split, own, row);
        convert_chunk<OUT>(v, sbuf, row, a.alpha, a.beta, a.ia, a.ib, a.use_beta, a.epi,
                           a.bias_row);
        fence_async_smem();
        named_bar_sync(1, 128);
        if (leader) {
            tma_store_3d(tmC, sbuf, a.m0, a.n0 + c0, a.b);
            bulk_commit();
            // every thread has read ring slot sl: refill it
            if (c0 + 32 * rslots < a.ncols) fetch(c0 / 32 + rslots);
        }
    }
    (void)lane;
    return st;
}

template <int KIND, int BN, bool A_MN, bool B_MN, int OUT, bool EPI_TMA, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
               const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmA2,
               const __grid_constant__ CUtensorMap tmB2,
               const __grid_constant__ CUtensorMap tmC,
               const TcParams p) {
    using C_ = Cfg<BN, KIND, EPI_TMA ? out_es(OUT) : 0, PAIR>;
    constexpr int BK = C_::BK, BOX = C_::BOX, STAGES = C_::STAGES;
    constexpr int B_ROWS = C_::B_ROWS;
    constexpr int TILE_M = PAIR ? 2 * BM : BM;           // output rows per tile
    constexpr int A_BYTES = C_::A_BYTES, B_BYTES = C_::B_BYTES;
    constexpr int STAGE_BYTES = C_::STAGE_BYTES;
    constexpr int UK = KT<KIND>::uk;
    constexpr int KSTEPS = BK / UK;
    constexpr uint32_t IDESC =
        make_idesc(KT<KIND>::cfmt, KT<KIND>::abfmt, A_MN ? 1 : 0, B_MN ? 1 : 0, TILE_M, BN);
    // half-width units of a split last wave: the same loads, N = BN/2
    constexpr uint32_t IDESC_HALF =
        make_idesc(KT<KIND>::cfmt, KT<KIND>::abfmt, A_MN ? 1 : 0, B_MN ? 1 : 0, TILE_M, BN / 2);
    constexpr uint32_t TMEM_COLS = C_::TMEM_COLS;
    constexpr bool CHUNKED = KIND == (int)Kind::TF32X3;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* epi = smem + STAGES * STAGE_BYTES;            // epilogue staging buffers
    uint64_t* full = reinterpret_cast<uint64_t*>(epi + C_::EPI_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* cbar = tempty + 2;                          // C chunk loaded, per buffer
    uint64_t* rbar = cbar + 2;                            // split partials staged, per ring slot
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 3);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* split_last = abort_flag + 1;            // epilogue: this part completes its tile

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // CTA pair: rank 0 (leader) issues the MMAs for both; each CTA loads its
    // own 128 rows of A and BN/2 columns of B and stores its 128 rows of C
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const int cta_id = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int n_ctas = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], PAIR ? 8 : 4);   // one arrival per epilogue warp (of both CTAs)
            mbar_init(&cbar[a], 1);
        }
        for (int a = 0; a < 3; a++) mbar_init(&rbar[a], 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if constexpr (C_::PLANES == 2) {
            prefetch_tmap(&tmA2);
            prefetch_tmap(&tmB2);
        }
        if constexpr (EPI_TMA) prefetch_tmap(&tmC);
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            tmem_alloc_pair(tmem_slot, TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    if constexpr (PAIR) cluster_sync();    // barriers of both CTAs initialised
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int total = p.total_units;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int u = cta_id; u < total; u += n_ctas) {
                const Unit un = unit_of(p, u);
                int b, tm, tn;
                decode_tile(un.t, p.tiles_m, p.tiles_n, b, tm, tn);
                const int m0 = tm * TILE_M + (int)rank * BM;
                // a half unit loads the full box from its half's first column
                // (each CTA of a pair from its quarter); the MMA reads the
                // leading BN/2 (or BN/4) columns
                const int n0 = tn * BN + (un.nh ? (un.nh - 1) * (BN / 2) : 0) +
                               (int)rank * (un.nh ? B_ROWS / 2 : B_ROWS);
                for (int kb = un.kb0; kb < un.kb1; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) goto producer_done;
                    uint8_t* sa = smem + stage * STAGE_BYTES;
                    uint8_t* sb = sa + A_BYTES;
                    const int k0 = kb * BK;
                    if constexpr (PAIR) {
                        // both CTAs' bytes complete on the leader's barrier
                        if (rank == 0) mbar_expect_tx(&full[stage], 2 * STAGE_BYTES);
                        const uint32_t bar0 = mapa_shared(&full[stage], 0);
                        load_operand_pair<A_MN, BM, BK, BOX>(sa, &tmA, bar0, m0, k0, b);
                        load_operand_pair<B_MN, B_ROWS, BK, BOX>(sb, &tmB, bar0, n0, k0, b);
                        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                        continue;
                    }
                    mbar_expect_tx(&full[stage], STAGE_BYTES);
                    load_operand<A_MN, BM, BK, BOX>(sa, &tmA, &full[stage], m0, k0, b);
                    load_operand<B_MN, BN, BK, BOX>(sb, &tmB, &full[stage], n0, k0, b);
                    if constexpr (C_::PLANES == 2) {
                        load_operand<A_MN, BM, BK, BOX>(sb + B_BYTES, &tmA2, &full[stage], m0, k0, b);
                        load_operand<B_MN, BN, BK, BOX>(sb + B_BYTES + A_BYTES, &tmB2, &full[stage], n0, k0, b);
                    }
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            // drain: wait until the MMA issuer has released every stage, so no
            // tcgen05.commit arrival is still travelling to this CTA's barriers
            // when it exits (for a pair they come from the other SM)
            for (int i = 0; i < STAGES; i++) {
                if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) break;
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
        producer_done:;
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0 && rank == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            // one accumulator per chunk of kc K blocks (a unit is one chunk
            // unless the kernel accumulates in chunks)
            for (int u = cta_id; u < total; u += n_ctas) {
                const Unit un = unit_of(p, u);
                const uint32_t idesc = un.nh ? IDESC_HALF : IDESC;
                for (int c0 = un.kb0; c0 < un.kb1; c0 += p.kc, local++) {
                const int c1 = min(c0 + p.kc, un.kb1);
                const int acc = local & 1;
                const uint32_t aphase = (local >> 1) & 1;
                if (!mbar_wait(&tempty[acc], aphase ^ 1u, abort_flag)) goto mma_done;
                tc_fence_after();
                const uint32_t d = tmem_base + acc * BN;
                for (int kb = c0; kb < c1; kb++) {
                    if (!mbar_wait(&full[stage], phase, abort_flag)) goto mma_done;
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
                    const uint32_t sb = sa + A_BYTES;
#pragma unroll
                    for (int ks = 0; ks < KSTEPS; ks++) {
                        const uint64_t ad = operand_desc<A_MN, BK, UK>(sa, ks);
                        const uint64_t bd = operand_desc<B_MN, BK, UK>(sb, ks);
                        const uint32_t accum = (kb != c0 || ks != 0) ? 1u : 0u;
                        if constexpr (KIND == (int)Kind::TF32X3) {
                            // small terms first: lo*hi, hi*lo, then hi*hi
                            const uint64_t ad2 = operand_desc<A_MN, BK, UK>(sb + B_BYTES, ks);
                            const uint64_t bd2 = operand_desc<B_MN, BK, UK>(sb + B_BYTES + A_BYTES, ks);
                            mma_tf32_ss(d, ad2, bd, idesc, accum);
                            mma_tf32_ss(d, ad, bd2, idesc, 1u);
                            mma_tf32_ss(d, ad, bd, idesc, 1u);
                        } else if constexpr (KIND == (int)Kind::TF32) {
                            mma_tf32_ss(d, ad, bd, idesc, accum);
                        } else if constexpr (KIND == (int)Kind::I8) {
                            if constexpr (PAIR) mma_i8_ss_pair(d, ad, bd, idesc, accum);
                            else mma_i8_ss(d, ad, bd, idesc, accum);
                        } else {
                            if constexpr (PAIR) mma_f16_ss_pair(d, ad, bd, idesc, accum);
                            else mma_f16_ss(d, ad, bd, idesc, accum);
                        }
                    }
                    if constexpr (PAIR) mma_commit_pair(&empty[stage], 0x3);
                    else mma_commit(&empty[stage]);
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
                if constexpr (PAIR) mma_commit_pair(&tfull[acc], 0x3);
                else mma_commit(&tfull[acc]);
                }
            }
        mma_done:;
        }
    } else {
        // ---------------- epilogue ----------------
        const int q = warp & 3;                 // TMEM lane quarter of this warp
        const int r_in_tile = q * 32 + lane;
        float alpha = p.alpha, beta = p.beta;
        int32_t ia = p.ialpha, ib = p.ibeta;
        if (p.alpha_dev) {
            if constexpr (OUT == kR32I) ia = *static_cast<const int32_t*>(p.alpha_dev);
            else alpha = *static_cast<const float*>(p.alpha_dev);
        }
        if (p.beta_dev) {
            if constexpr (OUT == kR32I) ib = *static_cast<const int32_t*>(p.beta_dev);
            else beta = *static_cast<const float*>(p.beta_dev);
        }
        const bool use_beta = OUT == kR32I ? ib != 0 : beta != 0.0f;
        if constexpr (EPI_TMA) {
            // Staged epilogue.  Per 32-column chunk: the leader TMA-loads the
            // chunk of C (for beta) into one of two staging buffers, every
            // thread converts its row from TMEM into the buffer in place, and
            // the leader TMA-stores the chunk (rows/columns past m/n are
            // clipped by TMA).  The leader waits for the store that last used
            // a buffer to finish reading it before refilling it.  Every sync
            // point is uniform over the 128 epilogue threads: a failed bounded
            // wait in any thread is combined with bar.red.and and all leave.
            constexpr int ES = out_es(OUT);
            const int et = threadIdx.x - 64;           // 0..127
            const bool leader = et == 0;
            uint32_t cphase = 0;                       // bit i: parity of cbar[i]
            uint32_t rphase = 0;                       // bit i: parity of rbar[i]
            int chunk = 0;
            int local = 0;
            bool ok = true;
            for (int u = cta_id; ok && u < total; u += n_ctas, local++) {
                const Unit un = unit_of(p, u);
                float run[CHUNKED ? BN : 1];
                const int nch = CHUNKED ? (un.kb1 - un.kb0 + p.kc - 1) / p.kc : 1;
                if constexpr (CHUNKED) {
                    for (int c = 0; c + 1 < nch; c++, local++) {
                        const int ca = local & 1;
                        ok = named_bar_and(1, 128,
                                           mbar_wait(&tfull[ca], (local >> 1) & 1, abort_flag));
                        if (!ok) break;
                        tc_fence_after();
                        fold_chunk<BN>(tmem_base + ((uint32_t)(q * 32) << 16) + ca * BN, run,
                                       c == 0);
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) release_acc(&tempty[ca], rank);
                    }
                    if (!ok) break;
                }
                const int acc = local & 1;
                const uint32_t aphase = (local >> 1) & 1;
                ok = named_bar_and(1, 128, mbar_wait(&tfull[acc], aphase, abort_flag));
                if (!ok) break;
                tc_fence_after();
                if constexpr (CHUNKED) {
                    if (nch > 1) add_run<BN>(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN, run);
                }
                int b, tm, tn;
                decode_tile(un.t, p.tiles_m, p.tiles_n, b, tm, tn);
                const int width = un.nh ? BN / 2 : BN;      // columns of this unit
                const int m0 = tm * TILE_M + (int)rank * BM,
                          n0 = tn * BN + (un.nh ? (un.nh - 1) * (BN / 2) : 0);
                const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
                const int ncols = min(width, p.n - n0);
                const float bias_row = load_bias(p, (long long)m0 + r_in_tile);
                if (un.part >= 0) {             // K-split unit: out of line
                    SplitArgs sa;
                    sa.work = p.work;
                    sa.counters = p.counters;
                    sa.epoch = p.epoch;
                    sa.split = p.split;
                    sa.tt = un.t - p.main_units;
                    sa.part = un.part;
                    sa.rank = (int)rank;
                    sa.ncols = ncols;
                    sa.taddr = taddr;
                    sa.m0 = m0;
                    sa.n0 = n0;
                    sa.b = b;
                    sa.alpha = alpha;
                    sa.beta = beta;
                    sa.bias_row = bias_row;
                    sa.ia = ia;
                    sa.ib = ib;
                    sa.epi = p.epi;
                    sa.use_beta = use_beta;
                    EpiState es{chunk, cphase, rphase, true};
                    es = split_unit_epilogue<BN, OUT, PAIR, C_::NEPI, C_::EPI_BUF,
                                             STAGES * STAGE_BYTES>(
                        sa, es, smem, epi, cbar, rbar, abort_flag, split_last, &tmC, r_in_tile,
                        lane, leader);
                    chunk = es.chunk;
                    cphase = es.cphase;
                    rphase = es.rphase;
                    ok = es.ok;
                    if (!ok) break;
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) release_acc(&tempty[acc], rank);
                    continue;
                }
                if (!use_beta) {
                    // C is not read: one barrier per chunk, and the TMEM load
                    // of chunk c+1 in flight while chunk c is converted.  The
                    // leader waits for the store of chunk c-1 to have read its
                    // buffer before the barrier, which then frees that buffer
                    // for chunk c+1; no wait inside can fail, so the barrier
                    // needs no vote.
                    uint32_t v[32], vn[32];
                    tmem_ld32(taddr, v);
                    tmem_wait_ld();
#pragma unroll 1
                    for (int c0 = 0; c0 < ncols; c0 += kEpiCols, chunk++) {
                        uint8_t* sbuf = epi + (chunk & 1) * C_::EPI_BUF;
                        const bool more = c0 + kEpiCols < ncols;
                        if (more) tmem_ld32(taddr + c0 + kEpiCols, vn);
                        convert_chunk<OUT>(v, sbuf, r_in_tile, alpha, beta, ia, ib, false, p.epi,
                                           bias_row);
                        fence_async_smem();
                        if (leader) bulk_wait_read<0>();
                        named_bar_sync(1, 128);
                        if (leader) {
                            tma_store_3d(&tmC, sbuf, m0, n0 + c0, b);
                            bulk_commit();
                        }
                        if (more) {
                            tmem_wait_ld();
#pragma unroll
                            for (int j = 0; j < 32; j++) v[j] = vn[j];
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) release_acc(&tempty[acc], rank);
                    continue;
                }
#pragma unroll 1
                for (int c0 = 0; c0 < ncols; c0 += kEpiCols, chunk++) {
                    const int buf = chunk & 1;
                    uint8_t* sbuf = epi + buf * C_::EPI_BUF;
                    if (leader) {
                        // C chunks are loaded one chunk ahead: a tile's first
                        // chunk here, chunk c+1 into the other buffer once the
                        // store that last used it has read it
                        if (c0 == 0) {
                            bulk_wait_read<1>();   // store of chunk-2 has read sbuf
                            mbar_expect_tx(&cbar[buf], C_::EPI_BUF);
                            tma_load_3d(sbuf, &tmC, &cbar[buf], m0, n0 + c0, b);
                        }
                        if (c0 + kEpiCols < ncols) {
                            bulk_wait_read<0>();   // store of chunk-1 has read the other buffer
                            mbar_expect_tx(&cbar[buf ^ 1], C_::EPI_BUF);
                            tma_load_3d(epi + (buf ^ 1) * C_::EPI_BUF, &tmC, &cbar[buf ^ 1], m0,
                                        n0 + c0 + kEpiCols, b);
                        }
                    }
                    uint32_t v[32];
                    tmem_ld32(taddr + c0, v);
                    bool w = mbar_wait(&cbar[buf], (cphase >> buf) & 1u, abort_flag);
                    cphase ^= 1u << buf;
                    tmem_wait_ld();
                    ok = named_bar_and(1, 128, w);
                    if (!ok) break;
                    convert_chunk<OUT>(v, sbuf, r_in_tile, alpha, beta, ia, ib, true, p.epi,
                                       bias_row);
                    fence_async_smem();
                    named_bar_sync(1, 128);
                    if (leader) {
                        tma_store_3d(&tmC, sbuf, m0, n0 + c0, b);
                        bulk_commit();
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) release_acc(&tempty[acc], rank);
            }
            if (leader) bulk_wait<0>();
        } else {
            int local = 0;
            // (the host never splits K for this epilogue: every unit is a tile)
            for (int u = cta_id; u < total; u += n_ctas, local++) {
                const Unit un = unit_of(p, u);
                float run[CHUNKED ? BN : 1];
                const int nch = CHUNKED ? (un.kb1 - un.kb0 + p.kc - 1) / p.kc : 1;
                bool fine = true;
                if constexpr (CHUNKED) {
                    for (int c = 0; c + 1 < nch; c++, local++) {
                        const int ca = local & 1;
                        if (!mbar_wait(&tfull[ca], (local >> 1) & 1, abort_flag)) { fine = false; break; }
                        tc_fence_after();
                        fold_chunk<BN>(tmem_base + ((uint32_t)(q * 32) << 16) + ca * BN, run,
                                       c == 0);
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) release_acc(&tempty[ca], rank);
                    }
                }
                if (!fine) break;
                const int acc = local & 1;
                const uint32_t aphase = (local >> 1) & 1;
                if (!mbar_wait(&tfull[acc], aphase, abort_flag)) break;
                tc_fence_after();
                if constexpr (CHUNKED) {
                    if (nch > 1) add_run<BN>(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN, run);
                }
                int b, tm, tn;
                decode_tile(un.t, p.tiles_m, p.tiles_n, b, tm, tn);
                const long long row = (long long)tm * TILE_M + (int)rank * BM + r_in_tile;
                const bool row_ok = row < p.m;
                const int width = un.nh ? BN / 2 : BN;      // columns of this unit
                const int n0 = tn * BN + (un.nh ? (un.nh - 1) * (BN / 2) : 0);
                const int nlim = min(p.n, n0 + width);
                const long long base = (long long)b * p.strideC + row;
                const float bias_row = load_bias(p, row);
                const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
                // beta * C: the old values of chunk c+1 are loaded while chunk c
                // is converted and stored, so C's read latency is paid once per
                // tile rather than once per column
                uint32_t old[32], old_next[32];
                auto fetch = [&](int c0, uint32_t (&dst)[32]) {
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        const int col = n0 + c0 + j;
                        dst[j] = (use_beta && row_ok && col < nlim)
                                     ? load_c<OUT>(p.C, base + (long long)col * p.ldc) : 0u;
                    }
                };
                fetch(0, old);
#pragma unroll 1
                for (int c0 = 0; c0 < width; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld32(taddr + c0, v);
                    if (c0 + 32 < width) fetch(c0 + 32, old_next);
                    tmem_wait_ld();
                    // the activation branch outside the unrolled loop (see
                    // convert_chunk_t): epi == 0 compiles to no activation code
                    if (row_ok && p.epi) {
#pragma unroll
                        for (int j = 0; j < 32; j++) {
                            const int col = n0 + c0 + j;
                            if (col < nlim)
                                store_out<OUT>(p.C, base + (long long)col * p.ldc, v[j], old[j],
                                               use_beta, alpha, beta, ia, ib, p.epi, bias_row);
                        }
                    } else if (row_ok) {
#pragma unroll
                        for (int j = 0; j < 32; j++) {
                            const int col = n0 + c0 + j;
                            if (col < nlim)
                                store_out<OUT>(p.C, base + (long long)col * p.ldc, v[j], old[j],
                                               use_beta, alpha, beta, ia, ib, 0, 0.f);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 32; j++) old[j] = old_next[j];
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) release_acc(&tempty[acc], rank);
            }
        }
    }

    tc_fence_before();
    if constexpr (PAIR) cluster_sync();   // neither CTA leaves while its pair may signal it
    else __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS);
        else tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---------------- host side ----------------

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
    static EncodeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
                cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeFn>(f);
    });
    return fn;
}

CUtensorMapDataType tmap_type(Kind k) {
    switch (k) {
    case Kind::F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    case Kind::BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    case Kind::I8: return CU_TENSOR_MAP_DATA_TYPE_UINT8;
    default: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    }
}

int elem_bytes(Kind k) {
    switch (k) {
    case Kind::F16: case Kind::BF16: return 2;
    case Kind::I8: return 1;
    default: return 4;
    }
}

// Tensor map for one operand.  `inner`/`outer` are the logical extents of
// the contiguous and strided dimensions, `ld` the stride between outer
// indices and `stride` the batch stride (elements).
bool make_tmap(CUtensorMap* tm, Kind kind, const void* base, long long inner,
               long long outer, long long ld, long long stride, int batch,
               int box_inner, int box_outer) {
    EncodeFn enc = encode_fn();
    if (!enc) return false;
    const int es = elem_bytes(kind);
    cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)batch};
    long long bstride = batch > 1 ? stride : ld * outer;
    if (bstride <= 0) bstride = ld * outer;
    cuuint64_t strides[2] = {(cuuint64_t)(ld * es), (cuuint64_t)(bstride * es)};
    // the batch stride of a single matrix is never used; keep it legal
    if (batch == 1) strides[1] = (strides[1] + 15) & ~cuuint64_t(15);
    cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(tm, tmap_type(kind), 3, const_cast<void*>(base), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Tensor map of C for the staged epilogue: dims {m, n, batch}, box {128
// rows, 32 columns, 1}, no swizzle (staging buffers are [column][row]).
bool make_cmap(CUtensorMap* tm, const GemmDesc& d) {
    EncodeFn enc = encode_fn();
    if (!enc) return false;
    CUtensorMapDataType t;
    int es;
    switch (d.Ctype) {
    case kR16F: t = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; es = 2; break;
    case kR16BF: t = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; es = 2; break;
    case kR32F: t = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; es = 4; break;
    case kR32I: t = CU_TENSOR_MAP_DATA_TYPE_INT32; es = 4; break;
    case kR8I: t = CU_TENSOR_MAP_DATA_TYPE_UINT8; es = 1; break;
    default: return false;
    }
    if ((reinterpret_cast<uintptr_t>(d.C) & 15u) || (d.ldc * es) % 16) return false;
    if (d.batch > 1 && (d.strideC <= 0 || (d.strideC * es) % 16)) return false;
    long long bstride = d.batch > 1 ? d.strideC : d.ldc * d.n;
    cuuint64_t dims[3] = {(cuuint64_t)d.m, (cuuint64_t)d.n, (cuuint64_t)d.batch};
    cuuint64_t strides[2] = {(cuuint64_t)(d.ldc * es),
                             ((cuuint64_t)(bstride * es) + 15) & ~cuuint64_t(15)};
    cuuint32_t box[3] = {(cuuint32_t)BM, (cuuint32_t)kEpiCols, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(tm, t, 3, d.C, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

struct Maps {
    CUtensorMap a, b, a2, b2, c;
    bool staged;            // C described by `c`: TMA-staged epilogue
    bool pair;              // CTA-pair (cta_group::2) kernel, 256-row tiles
    int sm_limit;           // most SMs to occupy (0 = all)
};

// Kinds and widths the CTA-pair kernel is built for.
// (each CTA holds BN/2 columns of B; an MN-major int8 swizzle row is 128
// columns wide, so int8 pairs need BN = 256)
constexpr bool pair_ok(int kind, int bn) {
    return (bn == 256 && kind == (int)Kind::I8) ||
           ((bn == 256 || bn == 128) && (kind == (int)Kind::F16 || kind == (int)Kind::BF16));
}

// K split of the last wave.  `tiles` tiles on `slots` persistent CTAs (or
// pairs) leave the last wave R = tiles % slots tiles; when R is at most half
// of the slots (and, by default, there is no full wave before it), each of
// those tiles is split into S = min(slots / R, 4)
// parts along K (each part at least 4 K blocks), so the last wave takes
// about 1/S of a tile's time.  `unit_bytes` is the workspace one part of
// one tile needs (0: this configuration does not split).  The part that
// completes a tile stages the other S-1 parts' 16 KB column chunks in the
// operand ring (`ring_bytes`), so S-1 chunks must fit there.  Without a
// workspace large enough, nothing is split.
void split_tail(TcParams& q, int tiles, int slots, size_t unit_bytes, size_t ring_bytes,
                bool halves_ok) {
    q.main_units = q.total_units = tiles;
    q.split = 1;
    q.tail_halves = 0;
    // A last wave after full waves that fills at most half of the CTAs:
    // each of its tiles becomes two half-width units, so the wave takes
    // about half a tile's time (no partial sums to combine).
    // ZBLAS_TAIL_HALVES=0 turns it off.
    {
        const char* th = getenv("ZBLAS_TAIL_HALVES");
        const int rem = slots > 0 ? tiles % slots : 0;
        if (halves_ok && !(th && th[0] == '0') && tiles >= slots && rem > 0 && 2 * rem <= slots) {
            q.tail_halves = 1;
            q.main_units = tiles - rem;
            q.total_units = tiles + rem;
            return;
        }
    }
    // ZBLAS_SPLIT_K: unset = split only a GEMM that is one sparse wave (fewer
    // tiles than half the CTAs: small m x n, long k); 1 = also the sparse
    // last wave after full waves (measured slower on 4096^3); 0 = never
    const char* sw = getenv("ZBLAS_SPLIT_K");
    if (sw && sw[0] == '0') return;
    const bool tails = sw && sw[0] == '1';
    if (!q.work || !q.counters || unit_bytes == 0 || slots <= 1) return;
    const int rem = tiles % slots;
    if (rem == 0 || 2 * rem > slots) return;
    if (tiles >= slots && !tails) return;
    int parts = slots / rem;
    if (parts > 4) parts = 4;
    while (parts > 1 && (q.k_blocks / parts < 4 || (size_t)(parts - 1) * 32 * BM * 4 > ring_bytes))
        parts--;
    if (parts < 2 || (size_t)rem * parts * unit_bytes > q.work_bytes) return;
    // two parts halve the main loop but not the completing part's epilogue,
    // which then also sums them: 1024 x 1024 x 4096 was slower split in two
    if (parts < 3 && !tails) return;
    q.split = parts;
    q.main_units = tiles - rem;
    q.total_units = q.main_units + rem * parts;
}

template <int KIND, int BN, bool A_MN, bool B_MN, int OUT, bool EPI_TMA, bool PAIR>
int launch_one(const Maps& m, const TcParams& p, cudaStream_t s) {
    using C_ = Cfg<BN, KIND, EPI_TMA ? out_es(OUT) : 0, PAIR>;
    auto kern = gemm_tc_kernel<KIND, BN, A_MN, B_MN, OUT, EPI_TMA, PAIR>;
    static std::atomic<unsigned long long> attr_set{0};   // one bit per device
    static int max_clusters[64] = {0};                    // co-resident pairs per device
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C_::SMEM);
        if (e != cudaSuccess) return (int)e;
        if constexpr (PAIR) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
            cudaLaunchConfig_t q = {};
            q.gridDim = dim3(2 * (num_sms() / 2));
            q.blockDim = dim3(kThreads);
            q.dynamicSmemBytes = C_::SMEM;
            cudaLaunchAttribute qa[1];
            qa[0].id = cudaLaunchAttributeClusterDimension;
            qa[0].val.clusterDim.x = 2;
            qa[0].val.clusterDim.y = 1;
            qa[0].val.clusterDim.z = 1;
            q.attrs = qa;
            q.numAttrs = 1;
            int nc = 0;
            e = cudaOccupancyMaxActiveClusters(&nc, kern, &q);
            if (e != cudaSuccess || nc <= 0) {
                cudaGetLastError();
                nc = num_sms() / 2;
            }
            max_clusters[dev & 63] = nc;
        }
        attr_set.fetch_or(bit);
    }
    int slots = PAIR ? (max_clusters[dev & 63] > 0 ? max_clusters[dev & 63] : num_sms() / 2)
                     : num_sms();
    if (m.sm_limit > 0) slots = std::min(slots, PAIR ? std::max(1, m.sm_limit / 2) : m.sm_limit);
    TcParams q = p;
    const int tiles = p.tiles_m * p.tiles_n * p.batch;
    // half units: each CTA's share of a half (BN/2, or BN/4 for a pair) must
    // be whole swizzle rows of an MN-major B tile
    constexpr int kHalfCols = PAIR ? BN / 4 : BN / 2;
    constexpr bool kHalvesOk = KIND != (int)Kind::TF32X3 && BN >= 128 &&
                               (!B_MN || kHalfCols % C_::BOX == 0);
    split_tail(q, tiles, slots, m.staged ? BN * BM * 4 * (PAIR ? 2 : 1) : 0,
               (size_t)C_::STAGES * C_::STAGE_BYTES, kHalvesOk);
    const int total = q.total_units;
    cudaError_t e;
    if constexpr (PAIR) {
        const int clusters = total < slots ? total : slots;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * clusters);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = C_::SMEM;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, kern, m.a, m.b, m.a2, m.b2, m.c, q);
    } else {
        const int grid = total < slots ? total : slots;
        kern<<<grid, kThreads, C_::SMEM, s>>>(m.a, m.b, m.a2, m.b2, m.c, q);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) note_launch();
    return e == cudaSuccess ? 0 : (int)e;
}

template <int KIND, int BN, bool A_MN, bool B_MN, int OUT>
int launch(const Maps& m, const TcParams& p, cudaStream_t s) {
    if constexpr (pair_ok(KIND, BN)) {
        if (m.pair)
            return m.staged ? launch_one<KIND, BN, A_MN, B_MN, OUT, true, true>(m, p, s)
                            : launch_one<KIND, BN, A_MN, B_MN, OUT, false, true>(m, p, s);
    }
    return m.staged ? launch_one<KIND, BN, A_MN, B_MN, OUT, true, false>(m, p, s)
                    : launch_one<KIND, BN, A_MN, B_MN, OUT, false, false>(m, p, s);
}

template <int KIND, int BN, int OUT>
int launch_majors(bool a_mn, bool b_mn, const Maps& m, const TcParams& p, cudaStream_t s) {
    if (a_mn && b_mn) return launch<KIND, BN, true, true, OUT>(m, p, s);
    if (a_mn) return launch<KIND, BN, true, false, OUT>(m, p, s);
    if (b_mn) return launch<KIND, BN, false, true, OUT>(m, p, s);
    return launch<KIND, BN, false, false, OUT>(m, p, s);
}

template <int KIND, int BN>
int launch_major(const GemmDesc& d, bool a_mn, bool b_mn, const Maps& m, const TcParams& p,
                 cudaStream_t s) {
    if constexpr (KIND == (int)Kind::I8) {
        if (d.Ctype == kR8I) return launch_majors<KIND, BN, kR8I>(a_mn, b_mn, m, p, s);
        if (d.Ctype != kR32I) return 1;
        return launch_majors<KIND, BN, kR32I>(a_mn, b_mn, m, p, s);
    } else if constexpr (KIND == (int)Kind::TF32X3 || KIND == (int)Kind::TF32) {
        if (d.Ctype != kR32F) return 1;
        return launch_majors<KIND, BN, kR32F>(a_mn, b_mn, m, p, s);
    } else {
        switch (d.Ctype) {
        case kR16F: return launch_majors<KIND, BN, kR16F>(a_mn, b_mn, m, p, s);
        case kR16BF: return launch_majors<KIND, BN, kR16BF>(a_mn, b_mn, m, p, s);
        case kR32F: return launch_majors<KIND, BN, kR32F>(a_mn, b_mn, m, p, s);
        default: return 1;
        }
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int num_sms() {
    int dev = 0;
    cudaGetDevice(&dev);
    static int cache[64] = {0};
    if (dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

int gemm_tc(const GemmDesc& d, cudaStream_t s) {
    if (getenv("ZBLAS_NO_TC")) return 1;
    if (d.m <= 0 || d.n <= 0 || d.k <= 0 || d.batch <= 0) return 1;
    const int es = elem_bytes(d.kind);
    // TMA: 16-byte aligned bases, 16-byte multiple strides
    const void* a_base = d.kind == Kind::TF32X3 ? (const void*)d.A_hi : d.A;
    const void* b_base = d.kind == Kind::TF32X3 ? (const void*)d.B_hi : d.B;
    if (!aligned16(a_base) || !aligned16(b_base)) return 1;
    if (d.kind == Kind::TF32X3 && (!aligned16(d.A_lo) || !aligned16(d.B_lo))) return 1;
    if ((d.lda * es) % 16 || (d.ldb * es) % 16) return 1;
    if (d.batch > 1 && ((d.strideA * es) % 16 || (d.strideB * es) % 16)) return 1;
    if (d.batch > 1 && (d.strideA <= 0 || d.strideB <= 0)) return 1;
    if (d.k > (1 << 30) || d.m > (1 << 30) || d.n > (1 << 30)) return 1;

    const bool a_mn = d.transa == 0;     // op(A)(i,l) = A[i + l*lda]: M contiguous
    const bool b_mn = d.transb != 0;     // op(B)(l,j) = B[j + l*ldb]: N contiguous
    const int bk = 128 / es, box = 128 / es;

    // Tile configuration.  fp16/bf16/int8: the candidate with the least
    // estimated time, waves * tile area / (SMs per tile * per-SM speed); the
    // speeds are B200 measurements of each configuration at 8192^3 (pair of
    // 256x256 tiles 1.00, single 128x256 0.90, single 128x128 0.69).  Pairs
    // need K >= 2048 bytes (short K: the pair's extra synchronisation
    // outweighs the halved B loads).  fp32 forms: 128 (or 64) wide tiles.
    const int sms = d.sm_limit > 0 ? std::min(num_sms(), std::max(2, d.sm_limit)) : num_sms();
    Maps maps;
    maps.pair = false;
    maps.sm_limit = d.sm_limit > 0 ? sms : 0;
    int BN = 128;
    if (d.kind == Kind::TF32X3 || d.kind == Kind::TF32) {
        const long long tiles256 = (long long)((d.m + BM - 1) / BM) * ((d.n + 255) / 256) * d.batch;
        BN = (d.kind == Kind::TF32 && tiles256 >= sms && d.n > 128) ? 256 : 128;
        if (d.kind == Kind::TF32X3) {
            const long long tiles128 = (long long)((d.m + BM - 1) / BM) * ((d.n + 127) / 128) * d.batch;
            if (tiles128 < sms) BN = 64;
        }
    } else {
        struct Cand { int bn; bool pair; double speed; };
        const Cand cands[3] = {{256, true, 1.00}, {256, false, 0.90}, {128, false, 0.69}};
        double best = 0.0;
        for (const Cand& c : cands) {
            if (c.pair && (getenv("ZBLAS_NO_PAIR") || (long long)d.k * es < 2048)) continue;
            const int rows = c.pair ? 2 * BM : BM;
            const long long tiles =
                (long long)((d.m + rows - 1) / rows) * ((d.n + c.bn - 1) / c.bn) * d.batch;
            const long long slots = c.pair ? sms / 2 : sms;
            const long long waves = (tiles + slots - 1) / slots;
            const double cost = (double)waves * rows * c.bn / ((c.pair ? 2.0 : 1.0) * c.speed);
            if (best == 0.0 || cost < best) {
                best = cost;
                BN = c.bn;
                maps.pair = c.pair;
            }
        }
    }
    if (const char* f = getenv("ZBLAS_GEMM_CFG")) {      // forced tile configuration
        if (pair_ok((int)d.kind, 256)) {
            const std::string cfg(f);
            if (cfg == "s128") { BN = 128; maps.pair = false; }
            if (cfg == "s256") { BN = 256; maps.pair = false; }
            if (cfg == "p128" && pair_ok((int)d.kind, 128)) { BN = 128; maps.pair = true; }
            if (cfg == "p256") { BN = 256; maps.pair = true; }
        }
    }
    const int b_rows = maps.pair ? BN / 2 : BN;
    CUtensorMap &ta = maps.a, &tb = maps.b, &ta2 = maps.a2, &tb2 = maps.b2;
    auto mk = [&](CUtensorMap* tm, const void* base, bool mn, long long mn_ext, long long ld,
                  long long stride, int rows) {
        if (mn) return make_tmap(tm, d.kind, base, mn_ext, d.k, ld, stride, d.batch, box, bk);
        return make_tmap(tm, d.kind, base, d.k, mn_ext, ld, stride, d.batch, bk, rows);
    };
    if (!mk(&ta, a_base, a_mn, d.m, d.lda, d.strideA, BM)) return 1;
    if (!mk(&tb, b_base, b_mn, d.n, d.ldb, d.strideB, b_rows)) return 1;
    if (d.kind == Kind::TF32X3) {
        if (!mk(&ta2, d.A_lo, a_mn, d.m, d.lda, d.strideA, BM)) return 1;
        if (!mk(&tb2, d.B_lo, b_mn, d.n, d.ldb, d.strideB, BN)) return 1;
    } else {
        ta2 = ta;
        tb2 = tb;
    }
    maps.staged = !getenv("ZBLAS_NO_TMA_EPILOGUE") && make_cmap(&maps.c, d);
    if (!maps.staged) maps.c = ta;

    TcParams p;
    p.m = d.m; p.n = d.n; p.k = d.k; p.batch = d.batch;
    p.tiles_m = maps.pair ? (d.m + 2 * BM - 1) / (2 * BM) : (d.m + BM - 1) / BM;
    p.tiles_n = (d.n + BN - 1) / BN;
    p.k_blocks = (d.k + bk - 1) / bk;
    p.ldc = d.ldc;
    p.strideC = d.strideC;
    p.C = d.C;
    p.out_type = d.Ctype;
    p.alpha = d.alpha; p.beta = d.beta;
    p.ialpha = d.ialpha; p.ibeta = d.ibeta;
    p.alpha_dev = d.alpha_dev; p.beta_dev = d.beta_dev;
    p.epi = d.kind == Kind::I8 ? 0 : d.epi;
    p.bias = d.bias;
    p.bias_type = d.bias_type;
    p.work = d.split_work;
    p.work_bytes = d.split_work_bytes;
    p.counters = d.split_counters;
    p.epoch = d.split_epoch & 0xffffffffffffull;
    p.main_units = p.total_units = p.tiles_m * p.tiles_n * p.batch;
    p.split = 1;
    p.tail_halves = 0;
    // 3xTF32: a fresh accumulator every 4 K blocks (128 of K)
    p.kc = d.kind == Kind::TF32X3 ? 4 : (p.k_blocks > 0 ? p.k_blocks : 1);

    switch (d.kind) {
    case Kind::F16:
        return BN == 256 ? launch_major<(int)Kind::F16, 256>(d, a_mn, b_mn, maps, p, s)
                         : launch_major<(int)Kind::F16, 128>(d, a_mn, b_mn, maps, p, s);
    case Kind::BF16:
        return BN == 256 ? launch_major<(int)Kind::BF16, 256>(d, a_mn, b_mn, maps, p, s)
                         : launch_major<(int)Kind::BF16, 128>(d, a_mn, b_mn, maps, p, s);
    case Kind::I8:
        return BN == 256 ? launch_major<(int)Kind::I8, 256>(d, a_mn, b_mn, maps, p, s)
                         : launch_major<(int)Kind::I8, 128>(d, a_mn, b_mn, maps, p, s);
    case Kind::TF32:
        return BN == 256 ? launch_major<(int)Kind::TF32, 256>(d, a_mn, b_mn, maps, p, s)
                         : launch_major<(int)Kind::TF32, 128>(d, a_mn, b_mn, maps, p, s);
    case Kind::TF32X3:
        return BN == 128 ? launch_major<(int)Kind::TF32X3, 128>(d, a_mn, b_mn, maps, p, s)
                         : launch_major<(int)Kind::TF32X3, 64>(d, a_mn, b_mn, maps, p, s);
    }
    return 1;
}

int gemm_tc_set_wait_limit(unsigned long long ns) { return set_unit_wait_limit(ns); }

int gemm_tc_error(bool clear) {
    int v = 0;
    cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(int));
    if (clear && v) {
        int z = 0;
        cudaMemcpyToSymbol(g_dev_error, &z, sizeof(int));
    }
    return v;
}

}  // namespace zl
