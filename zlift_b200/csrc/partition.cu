// partition.cu -- the multi-GPU partition layer (include/zlift_partition.h).
//
// Host code only: shard arithmetic, the per-shard calls into the same
// single-GPU entry points, and the one collective of the path (all-gather
// of C's column blocks for the N-split GEMM), issued through NCCL on the
// handle's stream so it follows the GEMM without a host round trip.
#include "fmha.h"
#include "gemm.h"

#include "../../include/zlift_cublas.h"
#include "../../include/zlift_partition.h"

#include <dlfcn.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <thread>
#include <vector>

namespace {

// The subset of NCCL's C API the layer uses (nccl.h, NCCL 2.x).
typedef struct { char internal[128]; } NcclUniqueId;
typedef void* NcclComm;
typedef int NcclResult;
enum { kNcclSuccess = 0, kNcclInProgress = 7 };
enum { kNcclInt8 = 0, kNcclInt32 = 2 };

struct Nccl {
    NcclResult (*get_unique_id)(NcclUniqueId*) = nullptr;
    NcclResult (*comm_init_rank)(NcclComm*, int, NcclUniqueId, int) = nullptr;
    NcclResult (*comm_destroy)(NcclComm) = nullptr;
    NcclResult (*comm_abort)(NcclComm) = nullptr;
    NcclResult (*comm_get_async_error)(NcclComm, NcclResult*) = nullptr;
    NcclResult (*all_gather)(const void*, void*, size_t, int, NcclComm, cudaStream_t) = nullptr;
    NcclResult (*broadcast)(const void*, void*, size_t, int, int, NcclComm, cudaStream_t) = nullptr;
    NcclResult (*group_start)() = nullptr;
    NcclResult (*group_end)() = nullptr;
    bool ok = false;
};

const Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = nullptr;
        if (const char* p = getenv("ZLIFT_NCCL_LIB")) h = dlopen(p, RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);   // already in the process
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        auto sym = [&](const char* s) { return dlsym(h, s); };
        n.get_unique_id = (decltype(n.get_unique_id))sym("ncclGetUniqueId");
        n.comm_init_rank = (decltype(n.comm_init_rank))sym("ncclCommInitRank");
        n.comm_destroy = (decltype(n.comm_destroy))sym("ncclCommDestroy");
        n.comm_abort = (decltype(n.comm_abort))sym("ncclCommAbort");
        n.comm_get_async_error = (decltype(n.comm_get_async_error))sym("ncclCommGetAsyncError");
        n.all_gather = (decltype(n.all_gather))sym("ncclAllGather");
        n.broadcast = (decltype(n.broadcast))sym("ncclBroadcast");
        n.group_start = (decltype(n.group_start))sym("ncclGroupStart");
        n.group_end = (decltype(n.group_end))sym("ncclGroupEnd");
        n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.comm_abort &&
               n.comm_get_async_error && n.all_gather && n.broadcast && n.group_start &&
               n.group_end;
    });
    return n;
}

int elem_size(int t) {
    switch (t) {
    case zl::kR16F: case zl::kR16BF: return 2;
    case zl::kR8I: return 1;
    default: return 4;
    }
}

// Per-communicator resources of the overlapped N-split: a second stream for
// the collectives and one event per sub-block (GEMM of sub-block s done on
// the handle's stream), plus the event the handle's stream waits on at the
// end.  Created on first use, released by zlift_part_comm_destroy.
struct Overlap {
    int device = -1;
    cudaStream_t stream = nullptr;
    std::vector<cudaEvent_t> gemm_done;
    cudaEvent_t gathered = nullptr;
};
std::mutex g_overlap_mu;
std::map<void*, Overlap> g_overlap;

Overlap* overlap_for(void* comm, int sub_blocks) {
    std::lock_guard<std::mutex> lock(g_overlap_mu);
    Overlap& o = g_overlap[comm];
    int dev = 0;
    cudaGetDevice(&dev);
    if (!o.stream) {
        if (cudaStreamCreateWithFlags(&o.stream, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&o.gathered, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            g_overlap.erase(comm);
            return nullptr;
        }
        o.device = dev;
    }
    if (o.device != dev) return nullptr;
    while ((int)o.gemm_done.size() < sub_blocks) {
        cudaEvent_t e;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        o.gemm_done.push_back(e);
    }
    return &o;
}

void release_overlap(void* comm) {
    std::lock_guard<std::mutex> lock(g_overlap_mu);
    auto it = g_overlap.find(comm);
    if (it == g_overlap.end()) return;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(it->second.device);
    for (cudaEvent_t e : it->second.gemm_done) cudaEventDestroy(e);
    if (it->second.gathered) cudaEventDestroy(it->second.gathered);
    if (it->second.stream) cudaStreamDestroy(it->second.stream);
    cudaSetDevice(cur);
    g_overlap.erase(it);
}

}  // namespace

extern "C" {

int zlift_part_range(long long total, int parts, int index, long long align, long long* begin,
                     long long* end) {
    if (!begin || !end || total < 0 || parts <= 0 || index < 0 || index >= parts || align <= 0)
        return 1;
    const long long units = (total + align - 1) / align;       // whole alignment units
    const long long base = units / parts, extra = units % parts;
    // the first `extra` ranks take one more unit
    const long long u0 = index * base + (index < extra ? index : extra);
    const long long u1 = u0 + base + (index < extra ? 1 : 0);
    long long b = u0 * align, e = u1 * align;
    if (b > total) b = total;
    if (e > total) e = total;
    *begin = b;
    *end = e;
    return 0;
}

int zlift_part_unique_id(void* id128) {
    const Nccl& n = nccl();
    if (!n.ok || !id128) return 1;
    NcclUniqueId id;
    NcclResult r = n.get_unique_id(&id);
    if (r != kNcclSuccess) return 100 + r;
    std::memcpy(id128, &id, sizeof id);
    return 0;
}

int zlift_part_comm_init(void** comm, int nranks, int rank, const void* id128) {
    const Nccl& n = nccl();
    if (!n.ok || !comm || !id128 || nranks <= 0 || rank < 0 || rank >= nranks) return 1;
    NcclUniqueId id;
    std::memcpy(&id, id128, sizeof id);
    NcclComm c = nullptr;
    NcclResult r = n.comm_init_rank(&c, nranks, id, rank);
    if (r != kNcclSuccess) return 100 + r;
    *comm = c;
    return 0;
}

int zlift_part_comm_destroy(void* comm) {
    const Nccl& n = nccl();
    if (!n.ok || !comm) return 1;
    release_overlap(comm);
    NcclResult r = n.comm_destroy(comm);
    return r == kNcclSuccess ? 0 : 100 + r;
}

int zlift_part_comm_wait(void* comm, void* stream, int timeout_ms) {
    const Nccl& n = nccl();
    if (!n.ok || !comm) return 1;
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        cudaError_t q = cudaStreamQuery(static_cast<cudaStream_t>(stream));
        if (q == cudaSuccess) return 0;
        if (q != cudaErrorNotReady) return 13;
        NcclResult err = kNcclSuccess;
        n.comm_get_async_error(comm, &err);
        if (err != kNcclSuccess && err != kNcclInProgress) {
            n.comm_abort(comm);
            release_overlap(comm);
            return 100 + err;
        }
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0).count();
        if (ms > timeout_ms) {
            n.comm_abort(comm);
            release_overlap(comm);
            return 200;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

int zlift_part_gemm_strided_batched_ex(void* handle, long long batch_begin, long long batch_end,
                                       int transa, int transb, int m, int n, int k,
                                       const void* alpha, const void* A, int Atype, int lda,
                                       long long strideA, const void* B, int Btype, int ldb,
                                       long long strideB, const void* beta, void* C, int Ctype,
                                       int ldc, long long strideC, int computeType) {
    if (batch_begin < 0 || batch_end < batch_begin || batch_end - batch_begin > 0x7fffffffLL)
        return CUBLAS_STATUS_INVALID_VALUE;
    const long long nb = batch_end - batch_begin;
    if (nb == 0) return CUBLAS_STATUS_SUCCESS;
    const char* a = static_cast<const char*>(A) + batch_begin * strideA * elem_size(Atype);
    const char* b = static_cast<const char*>(B) + batch_begin * strideB * elem_size(Btype);
    char* c = static_cast<char*>(C) + batch_begin * strideC * elem_size(Ctype);
    return cublasGemmStridedBatchedEx(handle, transa, transb, m, n, k, alpha, a, Atype, lda,
                                      strideA, b, Btype, ldb, strideB, beta, c, Ctype, ldc,
                                      strideC, (int)nb, computeType, 0);
}

int zlift_part_gemm_ex_nsplit(void* handle, void* comm, int nranks, int rank, int transa,
                              int transb, int m, int n, int k, const void* alpha, const void* A,
                              int Atype, int lda, const void* B_block, int Btype, int ldb,
                              const void* beta, void* C, int Ctype, int computeType) {
    if (nranks <= 0 || rank < 0 || rank >= nranks || m < 0 || n < 0) return 1;
    long long n0, n1;
    if (zlift_part_range(n, nranks, rank, 128, &n0, &n1)) return 1;
    const int es = elem_size(Ctype);
    char* c_block = static_cast<char*>(C) + n0 * (long long)m * es;
    int st = cublasGemmEx(handle, transa, transb, m, (int)(n1 - n0), k, alpha, A, Atype, lda,
                          B_block, Btype, ldb, beta, c_block, Ctype, m, computeType, 0);
    if (st) return st;
    if (nranks == 1) return 0;
    const Nccl& nc = nccl();
    if (!nc.ok || !comm) return 1;
    void* sv = nullptr;
    cublasGetStream_v2(handle, &sv);
    cudaStream_t s = static_cast<cudaStream_t>(sv);
    // equal blocks: one in-place all-gather; otherwise one broadcast per rank
    bool equal = true;
    long long b0, e0;
    zlift_part_range(n, nranks, 0, 128, &b0, &e0);
    for (int r = 1; r < nranks && equal; r++) {
        long long b, e;
        zlift_part_range(n, nranks, r, 128, &b, &e);
        equal = (e - b) == (e0 - b0);
    }
    const int dt = Ctype == zl::kR32I ? kNcclInt32 : kNcclInt8;
    const size_t unit = Ctype == zl::kR32I ? 1 : (size_t)es;   // elements of the NCCL type
    NcclResult r;
    if (equal) {
        const size_t count = (size_t)(e0 - b0) * (size_t)m * unit;
        r = nc.all_gather(c_block, C, count, dt, comm, s);
    } else {
        nc.group_start();
        r = kNcclSuccess;
        for (int q = 0; q < nranks && r == kNcclSuccess; q++) {
            long long b, e;
            zlift_part_range(n, nranks, q, 128, &b, &e);
            char* blk = static_cast<char*>(C) + b * (long long)m * es;
            const size_t count = (size_t)(e - b) * (size_t)m * unit;
            if (count) r = nc.broadcast(blk, blk, count, dt, q, comm, s);
        }
        NcclResult r2 = nc.group_end();
        if (r == kNcclSuccess) r = r2;
    }
    return r == kNcclSuccess ? 0 : 100 + r;
}

int zlift_part_nsplit_cols(long long n, int nranks, int rank, int sub_blocks, int s,
                           long long* begin, long long* end) {
    if (!begin || !end || n <= 0 || nranks <= 0 || rank < 0 || rank >= nranks || sub_blocks <= 0 ||
        s < 0 || s >= sub_blocks)
        return 1;
    const long long pieces = (long long)nranks * sub_blocks;
    if (n % pieces) return 1;
    const long long w = n / pieces;
    *begin = (long long)s * (n / sub_blocks) + (long long)rank * w;
    *end = *begin + w;
    return 0;
}

int zlift_part_gemm_ex_nsplit_overlap(void* handle, void* comm, int nranks, int rank,
                                      int sub_blocks, int transa, int transb, int m, int n,
                                      int k, const void* alpha, const void* A, int Atype,
                                      int lda, const void* B_cols, int Btype, int ldb,
                                      const void* beta, void* C, int Ctype, int computeType) {
    if (nranks <= 0 || rank < 0 || rank >= nranks || m < 0 || n <= 0 || sub_blocks <= 0 ||
        sub_blocks > 64)
        return 1;
    long long c0, c1;
    if (zlift_part_nsplit_cols(n, nranks, rank, sub_blocks, 0, &c0, &c1)) return 1;
    const long long w = c1 - c0;
    const int es = elem_size(Ctype);
    const int bes = elem_size(Btype);
    // sub-block s of op(B) in B_cols: w columns; transb = N: columns are
    // ldb apart, transb = T: rows of the stored matrix are adjacent
    const long long b_step = transb == 0 ? w * (long long)ldb : w;
    void* sv = nullptr;
    cublasGetStream_v2(handle, &sv);
    cudaStream_t s = static_cast<cudaStream_t>(sv);
    if (nranks == 1) {
        for (int sb = 0; sb < sub_blocks; sb++) {
            zlift_part_nsplit_cols(n, 1, 0, sub_blocks, sb, &c0, &c1);
            const int st = cublasGemmEx(handle, transa, transb, m, (int)w, k, alpha, A, Atype,
                                        lda, static_cast<const char*>(B_cols) + sb * b_step * bes,
                                        Btype, ldb, beta,
                                        static_cast<char*>(C) + c0 * (long long)m * es, Ctype, m,
                                        computeType, 0);
            if (st) return st;
        }
        return 0;
    }
    const Nccl& nc = nccl();
    if (!nc.ok || !comm) return 1;
    Overlap* ov = overlap_for(comm, sub_blocks);
    if (!ov) return 1;
    // leave SMs to NCCL's kernels, which run next to the GEMMs
    int target = 0;
    cublasGetSmCountTarget(handle, &target);
    int reserve = 16;
    if (const char* e = getenv("ZLIFT_PART_COMM_SMS")) reserve = atoi(e);
    const int sms = zl::num_sms();
    if (reserve > 0 && reserve < sms) cublasSetSmCountTarget(handle, sms - reserve);
    const int dt = Ctype == zl::kR32I ? kNcclInt32 : kNcclInt8;
    const size_t unit = Ctype == zl::kR32I ? 1 : (size_t)es;
    int rc = 0;
    for (int sb = 0; sb < sub_blocks && rc == 0; sb++) {
        zlift_part_nsplit_cols(n, nranks, rank, sub_blocks, sb, &c0, &c1);
        char* mine = static_cast<char*>(C) + c0 * (long long)m * es;
        rc = cublasGemmEx(handle, transa, transb, m, (int)w, k, alpha, A, Atype, lda,
                          static_cast<const char*>(B_cols) + sb * b_step * bes, Btype, ldb, beta,
                          mine, Ctype, m, computeType, 0);
        if (rc) break;
        // the gather of super-block sb (every rank's sub-block sb, in rank
        // order, in place) waits only for this GEMM on this rank; NCCL pairs
        // it with the same gather on the other ranks
        if (cudaEventRecord(ov->gemm_done[sb], s) != cudaSuccess ||
            cudaStreamWaitEvent(ov->stream, ov->gemm_done[sb], 0) != cudaSuccess) {
            cudaGetLastError();
            rc = 13;
            break;
        }
        char* super = static_cast<char*>(C) + (long long)sb * (n / sub_blocks) * m * es;
        NcclResult r = nc.all_gather(mine, super, (size_t)w * (size_t)m * unit, dt, comm,
                                     ov->stream);
        if (r != kNcclSuccess) rc = 100 + r;
    }
    cublasSetSmCountTarget(handle, target);
    // the handle's stream continues once the last gather has landed
    if (cudaEventRecord(ov->gathered, ov->stream) != cudaSuccess ||
        cudaStreamWaitEvent(s, ov->gathered, 0) != cudaSuccess) {
        cudaGetLastError();
        if (rc == 0) rc = 13;
    }
    return rc;
}

int zlift_part_flash_fwd(const void* params, unsigned bytes, int elem, long long pair_begin,
                         long long pair_end, void* stream) {
    if (pair_end <= pair_begin) return 0;
    return zl::flash_entry(params, bytes, elem, static_cast<cudaStream_t>(stream), pair_begin,
                           pair_end);
}

}  // extern "C"
