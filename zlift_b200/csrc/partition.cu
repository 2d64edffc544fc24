// partition.cu -- the multi-GPU partition layer (include/zlift_partition.h).
//
// Host code only: shard arithmetic, the per-shard calls into the same
// single-GPU entry points, and the one collective of the path (all-gather
// of C's column blocks for the N-split GEMM), issued through NCCL on the
// handle's stream so it follows the GEMM without a host round trip.
#include "fmha.h"
#include "gemm.h"
#include "ptx.cuh"

#include "../../include/zlift_cublas.h"
#include "../../include/zlift_partition.h"

#include <cuda.h>
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
    // copy-engine gather: one stream per peer (copies to different peers
    // run on different copy engines), each ending on its own event
    cudaStream_t peer_stream[8] = {};
    cudaEvent_t peer_done[8] = {};
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
    if (!o.peer_stream[0]) {
        for (int r = 0; r < 8; r++) {
            if (cudaStreamCreateWithFlags(&o.peer_stream[r], cudaStreamNonBlocking) != cudaSuccess ||
                cudaEventCreateWithFlags(&o.peer_done[r], cudaEventDisableTiming) != cudaSuccess) {
                cudaGetLastError();
                return nullptr;
            }
        }
    }
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
    for (int r = 0; r < 8; r++) {
        if (it->second.peer_done[r]) cudaEventDestroy(it->second.peer_done[r]);
        if (it->second.peer_stream[r]) cudaStreamDestroy(it->second.peer_stream[r]);
    }
    cudaSetDevice(cur);
    g_overlap.erase(it);
}

// ---- peer-memory gather (registered output buffers) ------------------------
//
// A registered C is mapped into every rank's address space (CUDA IPC); each
// rank then writes its column sub-blocks straight into the peers' C -- by
// copy-engine copies (cudaMemcpyAsync to the mapped peer address, one per
// peer and sub-block) or by a store kernel -- on the communicator's second
// stream, next to its own GEMM of the following sub-block, instead of an
// ncclAllGather.  Two flags per
// (step, source rank) in each rank's small flag array order it: READY (this
// rank's stream has reached the call, so its C may be overwritten) and DONE
// (the source has stored everything it owes this rank).  Every wait is
// bounded by the library's wait limit and records kErrWaitTimeout.

constexpr int kMaxRanks = 8;
// deadline of each exchange step of zlift_part_register_peer_buffer
constexpr int kRegisterTimeoutMs = 120000;
enum { kReady = 0, kDone = 1 };

struct PeerPtrs {
    uint4* dst[kMaxRanks];                  // peer copies of the same block (null: none)
    unsigned long long* flag[kMaxRanks];    // peer's flag word for this rank (null: self)
};

// flags[kind * kMaxRanks + source]: epoch of the last signal from `source`
__device__ __forceinline__ bool wait_flags(const volatile unsigned long long* flags, int kind,
                                           int nranks, int self, unsigned long long epoch) {
    const unsigned long long t0 = zl::globaltimer();
    for (int r = 0; r < nranks; r++) {
        if (r == self) continue;
        uint32_t spins = 0;
        while (flags[kind * kMaxRanks + r] < epoch) {
            if ((++spins & 255u) == 0 && zl::globaltimer() - t0 > zl::g_wait_limit_ns) {
                atomicCAS(&zl::g_dev_error, 0, (int)zl::kErrWaitTimeout);
                return false;
            }
        }
    }
    __threadfence_system();
    return true;
}

// One thread per peer: publish `epoch` in the peer's flag slot for this rank,
// after everything this GPU wrote before (fence at system scope).
__global__ void signal_peers_kernel(PeerPtrs pp, int nranks, unsigned long long epoch) {
    const int r = threadIdx.x;
    if (r >= nranks || !pp.flag[r]) return;
    __threadfence_system();
    *reinterpret_cast<volatile unsigned long long*>(pp.flag[r]) = epoch;
    __threadfence_system();
}

// Copies n16 16-byte words of this rank's block into every peer's C (the
// same offset), once every peer has signalled READY for `epoch`.
__global__ void __launch_bounds__(512) push_block_kernel(const uint4* __restrict__ src,
                                                         PeerPtrs pp, size_t n16, int nranks,
                                                         int self,
                                                         const unsigned long long* flags,
                                                         unsigned long long epoch) {
    __shared__ int go;
    if (threadIdx.x == 0) go = wait_flags(flags, kReady, nranks, self, epoch) ? 1 : 0;
    __syncthreads();
    if (!go) return;
    // four 16-byte words in flight per thread
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n16; i += 4 * stride) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; u++) v[u] = src[i + u * stride];
#pragma unroll
        for (int r = 0; r < kMaxRanks; r++)
            if (pp.dst[r]) {
#pragma unroll
                for (int u = 0; u < 4; u++) pp.dst[r][i + u * stride] = v[u];
            }
    }
    for (; i < n16; i += stride) {
        const uint4 v = src[i];
#pragma unroll
        for (int r = 0; r < kMaxRanks; r++)
            if (pp.dst[r]) pp.dst[r][i] = v;
    }
    __threadfence_system();
}

// Waits (one thread) until every peer has signalled DONE (or READY) for `epoch`.
__global__ void wait_flags_kernel(const unsigned long long* flags, int kind, int nranks,
                                  int self, unsigned long long epoch) {
    if (threadIdx.x == 0) wait_flags(flags, kind, nranks, self, epoch);
}

struct PeerBuf {
    int nranks = 0, rank = 0, device = -1;
    char* C = nullptr;
    size_t bytes = 0;
    char* peer_C[kMaxRanks] = {};              // peers' C in this address space (self: C)
    void* peer_base[kMaxRanks] = {};           // opened IPC mappings of C's allocation
    unsigned long long* flags = nullptr;       // this rank's [2][kMaxRanks] flag words
    unsigned long long* peer_flags[kMaxRanks] = {};   // peers' flag arrays
    unsigned long long epoch = 0;
};
std::mutex g_peer_mu;
std::map<std::pair<void*, void*>, PeerBuf> g_peer;     // (comm, C)

using AddrRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
AddrRangeFn addr_range_fn() {
    static AddrRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) ==
                cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<AddrRangeFn>(f);
        else
            cudaGetLastError();
    });
    return fn;
}

void close_peer_buf(PeerBuf& b) {
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(b.device);
    for (int r = 0; r < kMaxRanks; r++) {
        if (b.peer_base[r]) cudaIpcCloseMemHandle(b.peer_base[r]);
        if (b.peer_flags[r] && r != b.rank) cudaIpcCloseMemHandle(b.peer_flags[r]);
    }
    if (b.flags) cudaFree(b.flags);
    cudaGetLastError();
    cudaSetDevice(cur);
}

void release_peer_bufs(void* comm) {
    std::lock_guard<std::mutex> lock(g_peer_mu);
    for (auto it = g_peer.begin(); it != g_peer.end();) {
        if (it->first.first == comm) {
            close_peer_buf(it->second);
            it = g_peer.erase(it);
        } else {
            ++it;
        }
    }
}

PeerBuf* find_peer_buf(void* comm, void* C) {
    std::lock_guard<std::mutex> lock(g_peer_mu);
    auto it = g_peer.find({comm, C});
    return it == g_peer.end() ? nullptr : &it->second;
}

}  // namespace

namespace zl {
int part_error(bool clear) {
    int v = 0;
    cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(int));
    if (clear && v) {
        int z = 0;
        cudaMemcpyToSymbol(g_dev_error, &z, sizeof(int));
    }
    return v;
}
int part_set_wait_limit(unsigned long long ns) { return set_unit_wait_limit(ns); }
}  // namespace zl

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
    release_peer_bufs(comm);
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
            release_peer_bufs(comm);
            return 100 + err;
        }
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0).count();
        if (ms > timeout_ms) {
            n.comm_abort(comm);
            release_overlap(comm);
            release_peer_bufs(comm);
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

int zlift_part_register_peer_buffer(void* comm, int nranks, int rank, void* C, size_t bytes) {
    const Nccl& nc = nccl();
    if (!nc.ok || !comm || !C || bytes == 0 || nranks <= 1 || nranks > kMaxRanks || rank < 0 ||
        rank >= nranks)
        return 1;
    if (find_peer_buf(comm, C)) return 0;                 // already registered
    AddrRangeFn range = addr_range_fn();
    if (!range) return 1;
    CUdeviceptr base = 0;
    size_t alloc = 0;
    if (range(&base, &alloc, reinterpret_cast<CUdeviceptr>(C)) != CUDA_SUCCESS) return 1;
    const unsigned long long off = reinterpret_cast<CUdeviceptr>(C) - base;
    if (off + bytes > alloc) return 1;
    struct Info {
        cudaIpcMemHandle_t c, f;
        unsigned long long off, bytes;
    };
    PeerBuf b;
    b.nranks = nranks;
    b.rank = rank;
    cudaGetDevice(&b.device);
    b.C = static_cast<char*>(C);
    b.bytes = bytes;
    Info mine{};
    int rc = 0;
    if (cudaMalloc(&b.flags, 2 * kMaxRanks * sizeof(unsigned long long)) != cudaSuccess ||
        cudaMemset(b.flags, 0, 2 * kMaxRanks * sizeof(unsigned long long)) != cudaSuccess ||
        cudaIpcGetMemHandle(&mine.c, reinterpret_cast<void*>(base)) != cudaSuccess ||
        cudaIpcGetMemHandle(&mine.f, b.flags) != cudaSuccess)
        rc = 13;
    mine.off = off;
    mine.bytes = bytes;
    // exchange the handles through the communicator (in-place all-gather of
    // one Info per rank), then open every peer's mappings
    Info* dinfo = nullptr;
    cudaStream_t st = nullptr;
    std::vector<Info> all(nranks);
    if (cudaMalloc(&dinfo, sizeof(Info) * nranks) != cudaSuccess ||
        cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) {
        rc = 13;
    } else if (cudaMemset(dinfo, 0, sizeof(Info) * nranks) != cudaSuccess ||
               (rc == 0 && cudaMemcpy(dinfo + rank, &mine, sizeof(Info),
                                      cudaMemcpyHostToDevice) != cudaSuccess)) {
        rc = 13;
    }
    // Every rank takes part in both all-gathers, even one that failed above
    // (it sends zeros, then its error code), so no rank waits for it.  Each
    // gather is waited for with a deadline: a rank that never arrives aborts
    // the communicator (200) instead of blocking here.  A gather that cannot
    // even be enqueued leaves the communicator in an unknown state and
    // aborts it too, so a result >= 100 always means "aborted".
    bool aborted = false;
    auto gather = [&](const void* send, void* recv, size_t count) {
        NcclResult r = nc.all_gather(send, recv, count, kNcclInt8, comm, st);
        if (r != kNcclSuccess) {
            nc.comm_abort(comm);
            release_overlap(comm);
            release_peer_bufs(comm);
            aborted = true;
            rc = 100 + r;
            return;
        }
        const int w = zlift_part_comm_wait(comm, st, kRegisterTimeoutMs);
        if (w >= 100) aborted = true;
        if (w && rc == 0) rc = w;
    };
    if (dinfo && st) {
        gather(dinfo + rank, dinfo, sizeof(Info));
        if (!aborted && cudaMemcpy(all.data(), dinfo, sizeof(Info) * nranks,
                                   cudaMemcpyDeviceToHost) != cudaSuccess && rc == 0)
            rc = 13;
    }
    for (int p = 0; rc == 0 && p < nranks; p++) {
        if (p == rank) {
            b.peer_C[p] = b.C;
            continue;
        }
        if (all[p].bytes != bytes) { rc = 1; break; }
        void* pb = nullptr;
        void* pf = nullptr;
        if (cudaIpcOpenMemHandle(&pb, all[p].c, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            rc = 13;
            break;
        }
        b.peer_base[p] = pb;
        if (cudaIpcOpenMemHandle(&pf, all[p].f, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            rc = 13;
            break;
        }
        b.peer_flags[p] = static_cast<unsigned long long*>(pf);
        b.peer_C[p] = static_cast<char*>(pb) + all[p].off;
    }
    // agreement: the buffer is registered on every rank or on none (each
    // rank's status, gathered; the first nonzero one is every rank's result)
    if (dinfo && st && !aborted) {
        std::vector<int> codes(nranks, 0);
        int* dcodes = reinterpret_cast<int*>(dinfo);
        const int mine_rc = rc;
        if (cudaMemcpy(dcodes + rank, &mine_rc, sizeof(int), cudaMemcpyHostToDevice) !=
                cudaSuccess && rc == 0)
            rc = 13;
        gather(dcodes + rank, dcodes, sizeof(int));
        if (!aborted && cudaMemcpy(codes.data(), dcodes, sizeof(int) * nranks,
                                   cudaMemcpyDeviceToHost) == cudaSuccess) {
            for (int p = 0; p < nranks && rc == 0; p++)
                if (codes[p]) rc = codes[p];
        } else if (rc == 0) {
            rc = 13;
        }
    }
    if (st) cudaStreamDestroy(st);
    if (dinfo) cudaFree(dinfo);
    if (rc) {
        cudaGetLastError();
        close_peer_buf(b);
        return rc;
    }
    std::lock_guard<std::mutex> lock(g_peer_mu);
    g_peer[{comm, C}] = b;
    return 0;
}

int zlift_part_unregister_peer_buffer(void* comm, void* C) {
    std::lock_guard<std::mutex> lock(g_peer_mu);
    auto it = g_peer.find({comm, C});
    if (it == g_peer.end()) return 1;
    cudaDeviceSynchronize();
    close_peer_buf(it->second);
    g_peer.erase(it);
    return 0;
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
    // a registered C (zlift_part_register_peer_buffer) is gathered by peer
    // stores, else by NCCL
    PeerBuf* pbuf = find_peer_buf(comm, C);
    const size_t sub_bytes = (size_t)w * (size_t)m * es;
    if (pbuf && (pbuf->nranks != nranks || pbuf->rank != rank || sub_bytes % 16 ||
                 (reinterpret_cast<uintptr_t>(C) & 15) ||
                 (size_t)n * (size_t)m * es > pbuf->bytes))
        pbuf = nullptr;
    // registered C: the sub-blocks go to the peers by copy-engine copies
    // (default; no SM is taken from the GEMM) or by a store kernel
    // (ZLIFT_PART_GATHER=sm, ZLIFT_PART_PUSH_SMS CTAs)
    const char* gmode = getenv("ZLIFT_PART_GATHER");
    const bool by_ce = pbuf && !(gmode && gmode[0] == 's');
    // leave SMs to the gather's kernels, which run next to the GEMMs
    int target = 0;
    cublasGetSmCountTarget(handle, &target);
    int reserve = pbuf ? (by_ce ? 0 : 32) : 16;
    if (const char* e = getenv(pbuf ? "ZLIFT_PART_PUSH_SMS" : "ZLIFT_PART_COMM_SMS"))
        if (!by_ce) reserve = atoi(e);
    const int sms = zl::num_sms();
    if (reserve > 0 && reserve < sms) cublasSetSmCountTarget(handle, sms - reserve);
    if (pbuf) {
        const unsigned long long epoch = ++pbuf->epoch;
        PeerPtrs sig{};
        for (int r = 0; r < nranks; r++)
            if (r != rank) sig.flag[r] = pbuf->peer_flags[r] + kReady * kMaxRanks + rank;
        // this rank's C may be overwritten once its stream has reached here
        signal_peers_kernel<<<1, 32, 0, s>>>(sig, nranks, epoch);
        int rc = cudaGetLastError() == cudaSuccess ? 0 : 13;
        const int ctas = reserve > 0 && reserve < sms ? reserve : 16;
        bool ready_waited = false;
        for (int sb = 0; sb < sub_blocks && rc == 0; sb++) {
            zlift_part_nsplit_cols(n, nranks, rank, sub_blocks, sb, &c0, &c1);
            const size_t off = (size_t)c0 * (size_t)m * es;
            rc = cublasGemmEx(handle, transa, transb, m, (int)w, k, alpha, A, Atype, lda,
                              static_cast<const char*>(B_cols) + sb * b_step * bes, Btype, ldb,
                              beta, pbuf->C + off, Ctype, m, computeType, 0);
            if (rc) break;
            if (cudaEventRecord(ov->gemm_done[sb], s) != cudaSuccess ||
                cudaStreamWaitEvent(ov->stream, ov->gemm_done[sb], 0) != cudaSuccess) {
                rc = 13;
                break;
            }
            if (by_ce) {
                // the copies may start once every peer is READY (one wait per
                // call, on the second stream, which every peer stream follows)
                if (!ready_waited) {
                    wait_flags_kernel<<<1, 32, 0, ov->stream>>>(pbuf->flags, kReady, nranks, rank,
                                                               epoch);
                    if (cudaGetLastError() != cudaSuccess) { rc = 13; break; }
                    zl::note_launch();
                    ready_waited = true;
                }
                if (cudaEventRecord(ov->gemm_done[sb], ov->stream) != cudaSuccess) {
                    rc = 13;
                    break;
                }
                for (int r = 0; r < nranks && rc == 0; r++) {
                    if (r == rank) continue;
                    if (cudaStreamWaitEvent(ov->peer_stream[r], ov->gemm_done[sb], 0) !=
                            cudaSuccess ||
                        cudaMemcpyAsync(pbuf->peer_C[r] + off, pbuf->C + off, sub_bytes,
                                        cudaMemcpyDeviceToDevice, ov->peer_stream[r]) !=
                            cudaSuccess)
                        rc = 13;
                }
                continue;
            }
            PeerPtrs pp{};
            for (int r = 0; r < nranks; r++)
                if (r != rank) pp.dst[r] = reinterpret_cast<uint4*>(pbuf->peer_C[r] + off);
            push_block_kernel<<<ctas, 512, 0, ov->stream>>>(
                reinterpret_cast<const uint4*>(pbuf->C + off), pp, sub_bytes / 16, nranks, rank,
                pbuf->flags, epoch);
            if (cudaGetLastError() != cudaSuccess) rc = 13;
            else zl::note_launch();
        }
        cublasSetSmCountTarget(handle, target);
        if (by_ce) {
            // the DONE signal follows every peer stream's copies
            for (int r = 0; r < nranks && rc == 0; r++) {
                if (r == rank) continue;
                if (cudaEventRecord(ov->peer_done[r], ov->peer_stream[r]) != cudaSuccess ||
                    cudaStreamWaitEvent(ov->stream, ov->peer_done[r], 0) != cudaSuccess)
                    rc = 13;
            }
        }
        // tell every peer that all of its columns from this rank have landed;
        // a call that failed part-way does not, so its peers' bounded waits
        // run out and report the failure instead of using partial columns
        if (rc == 0) {
            PeerPtrs done{};
            for (int r = 0; r < nranks; r++)
                if (r != rank) done.flag[r] = pbuf->peer_flags[r] + kDone * kMaxRanks + rank;
            signal_peers_kernel<<<1, 32, 0, ov->stream>>>(done, nranks, epoch);
            if (cudaGetLastError() != cudaSuccess) rc = 13;
        }
        // the handle's stream continues once this rank's stores are out and
        // every peer's have arrived
        if (cudaEventRecord(ov->gathered, ov->stream) != cudaSuccess ||
            cudaStreamWaitEvent(s, ov->gathered, 0) != cudaSuccess) {
            if (rc == 0) rc = 13;
        }
        wait_flags_kernel<<<1, 32, 0, s>>>(pbuf->flags, kDone, nranks, rank, epoch);
        if (cudaGetLastError() != cudaSuccess && rc == 0) rc = 13;
        zl::note_launch(3);
        return rc;
    }
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
