// Host side of libcolizig_cuda.so: the device context, the keyed resident
// weight store behind colizig_cuda_matmul_fp8, the MoE layer registry and every
// exported entry point of include/colizig_cuda.h.
//
// The reference keeps one global device context guarded by the caller's
// spinlock (gpu.zig:51-62) and an LRU of VRAM slots (colizig_cuda.cu:80-169).
// Here the context is guarded by a mutex inside the library, MoE weights are
// registered once into resident HBM (no per-call upload), and every entry
// point saves/restores the host MXCSR like the reference's CsrGuard
// (colizig_cuda.cu:22-29): the CUDA runtime may turn on flush-to-zero on the
// calling thread, which would silently change the caller's CPU float math.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <climits>
#include <list>
#include <map>
#include <mutex>
#include <thread>
#include <unordered_map>
#include <tuple>
#include <vector>

#if defined(__x86_64__) || defined(_M_X64)
#include <xmmintrin.h>
#define CZ_HAVE_MXCSR 1
#endif

#include "../../include/colizig_cuda.h"
#include "cz_common.cuh"
#include "cz_internal.h"

#define CZ_EXPORT extern "C" __attribute__((visibility("default")))

namespace {

struct CsrGuard {
#ifdef CZ_HAVE_MXCSR
    unsigned saved;
    CsrGuard() : saved(_mm_getcsr()) {}
    ~CsrGuard() { _mm_setcsr(saved); }
#endif
};

// Pinned host staging (grown on demand, freed at shutdown), mapped into the
// device's address space: `dev` is the address kernels write it through.
struct HostBuf {
    void* p = nullptr;
    void* dev = nullptr;
    size_t cap = 0;
    bool ensure(size_t need) {
        if (cap >= need && p) return true;
        if (p) cudaFreeHost(p);
        p = dev = nullptr;
        cap = 0;
        if (need == 0) need = 16;
        if (cudaHostAlloc(&p, need, cudaHostAllocMapped) != cudaSuccess) {
            p = nullptr;
            return false;
        }
        if (cudaHostGetDevicePointer(&dev, p, 0) != cudaSuccess) {
            cudaFreeHost(p);
            p = nullptr;
            return false;
        }
        cap = need;
        return true;
    }
    void release() {
        if (p) cudaFreeHost(p);
        p = dev = nullptr;
        cap = 0;
    }
};

struct DevBuf {
    void* p = nullptr;
    size_t cap = 0;
    bool ensure(size_t need) {
        if (cap >= need && p) return true;
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        if (need == 0) need = 16;
        if (cudaMalloc(&p, need) != cudaSuccess) {
            p = nullptr;
            return false;
        }
        cap = need;
        return true;
    }
    // Like ensure, but a growth takes at least 1.5x the old capacity: buffers sized
    // by data-dependent counts (the sharded exchange) then reallocate, and so
    // synchronise the device, only a few times.
    bool ensure_grow(size_t need) {
        if (cap >= need && p) return true;
        const size_t want = need > cap + cap / 2 ? need : cap + cap / 2;
        return ensure(want) || ensure(need);
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
    }
    template <class T>
    T* as() const {
        return reinterpret_cast<T*>(p);
    }
};

struct Keyed {
    void* w = nullptr;
    void* s = nullptr;
    size_t wb = 0, sb = 0;
    std::list<uint64_t>::iterator lru;
};

struct MoeLayer {
    colizig_moe_dims d{};
    void* mem = nullptr;
    size_t bytes = 0;
    float* router = nullptr;
    uint8_t *gate_w = nullptr, *up_w = nullptr, *down_w = nullptr;
    float *gate_s = nullptr, *up_s = nullptr, *down_s = nullptr;
    uint8_t *sh_gate_w = nullptr, *sh_up_w = nullptr, *sh_down_w = nullptr;
    float *sh_gate_s = nullptr, *sh_up_s = nullptr, *sh_down_s = nullptr;
    float* sh_gate = nullptr;
    int e_lo = 0, e_hi = 0;     // routed experts held here (all of them without expert parallelism)
    int shared_here = 0;        // the shared expert's weights are held (and computed) here
    bool ep = false;            // outputs are summed over the expert-parallel group after each forward
    cz::PrefillLayer pf{};      // the prefill kernels' view (tensor maps with 128-byte swizzle)
    bool pf_ok = false;
    CUtensorMap gate_map{}, up_map{}, sh_gate_map{}, sh_up_map{};  // decode views of the gate/up weights
    int gu_kb = 0;              // depth of those boxes (0 = 2D maps)
    uint64_t serial = 0;        // distinct for every registration (keys the captured host-call graphs)
    // BF16 shared expert (the reference's NativeMatrix, moe.zig:297-338): its own
    // allocation, held and computed on every rank; the routed kernels see d with
    // shared_inter = 0 and it runs beside them (moe_shared_bf16.cu)
    uint32_t shb_si = 0;
    void* shb_mem = nullptr;
    uint16_t *shb_g = nullptr, *shb_u = nullptr, *shb_d = nullptr;  // [SI][H], [SI][H], [H][SI]
    float* shb_gate = nullptr;                                      // [H]
};

// A host-pointer decode call captured as a CUDA graph (token upload, decode
// launches, one copy of the results back): the key holds everything the
// captured nodes point at or depend on.
struct HostGraphKey {
    uint32_t layer;
    uint64_t serial;
    int T, bf16, has_idx, has_gates;
    const void *io_x, *io_res, *io_host, *io_xh, *logits, *hrows, *sync;
    bool operator<(const HostGraphKey& o) const {
        return std::tie(layer, serial, T, bf16, has_idx, has_gates, io_x, io_res, io_host, io_xh, logits, hrows, sync) <
               std::tie(o.layer, o.serial, o.T, o.bf16, o.has_idx, o.has_gates, o.io_x, o.io_res, o.io_host, o.io_xh,
                        o.logits, o.hrows, o.sync);
    }
};

struct Ctx {
    bool inited = false;
    int dev = 0;
    int num_sms = 0;
    char name[192] = {0};
    cudaStream_t stream = nullptr;
    // legacy matmul scratch
    DevBuf d_x, d_y, d_w, d_s;
    // keyed resident store
    std::unordered_map<uint64_t, Keyed> keyed;
    std::list<uint64_t> lru;  // front = most recent
    size_t budget = 0, used = 0;
    uint64_t hits = 0, misses = 0, uploaded = 0;
    // MoE
    std::map<uint32_t, MoeLayer> layers;
    DevBuf logits, hrows, io_x, io_out, io_res, ones, pf_scratch;
    DevBuf shb_scratch;  // BF16 shared expert: gate/up rows and sigmoid gates of the call's tokens
    HostBuf io_host;  // pinned staging of io_res (host-pointer forward, up to kHostStageCap bytes)
    HostBuf mm_xh, mm_yh;  // pinned staging of colizig_cuda_matmul_fp8's x and y (up to kHostStageCap bytes)
    HostBuf io_xh;    // pinned staging of the tokens (host-pointer forward, up to kHostStageCap bytes)
    uint32_t* sync = nullptr;
    // expert parallelism (one process per GPU)
    bool ep_on = false;
    int ep_rank = 0, ep_world = 1;
    ncclComm_t ep_comm = nullptr;
    int ep_timeout_ms = 60000;  // watched host waits while a communicator is active (<= 0: unwatched)
    bool ep_aborted = false;    // the communicator was aborted; EP calls return -9 until re-initialised
    // decode combine inside the kernel: this rank's receive buffer (kEpRecvBytes,
    // zeroed), every rank's slot area as mapped here, the peers' IPC mappings
    void* ep_recv = nullptr;
    void* ep_peer_map[cz::kEpMaxRanks] = {};
    unsigned long long* ep_slots[cz::kEpMaxRanks] = {};
    bool ep_p2p = false;       // set up on every rank
    bool ep_p2p_use = true;    // colizig_cuda_ep_set_combine (the same on every rank)
    // sharded expert parallelism (prefill): routing of this rank's tokens, exchange buffers
    DevBuf sh_idx, sh_gates, sh_xn, sh_slot, sh_counts, sh_allc, sh_tmp, sh_send, sh_recv, sh_x, sh_ridx, sh_rgates,
        sh_part, sh_back;
    // failure-path tests: the next decode launch holds back router row 0's logits
    // and gives up its waits after dbg_spin_limit polls (one launch, then cleared)
    int dbg_hold = 0;
    uint32_t dbg_spin_limit = 0;
    // host-pointer decode calls: captured graphs, and the keys seen once (a key's
    // first call runs directly, which also makes every allocation it needs)
    std::map<HostGraphKey, cudaGraphExec_t> host_graphs;
    std::map<HostGraphKey, int> host_seen;
    uint64_t next_serial = 1;
    // kernel timer (benchmarks): CUDA event pairs around the dominant launches
    std::vector<cudaEvent_t> tm_ev;
    std::vector<int> tm_kind;
    int tm_n = 0;  // pairs recorded
    bool tm_overflow = false;
};

// NCCL is resolved at run time (dlopen of libnccl.so.2): the library loads without
// it, and a process that already loaded NCCL (torch does) shares that copy.
struct NcclApi {
    void* h = nullptr;
    ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*groupStart)() = nullptr;
    ncclResult_t (*groupEnd)() = nullptr;
    // optional (the watchdog uses them when present)
    ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    bool load() {
        if (h) return true;
        void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) return false;
        getUniqueId = reinterpret_cast<decltype(getUniqueId)>(dlsym(lib, "ncclGetUniqueId"));
        commInitRank = reinterpret_cast<decltype(commInitRank)>(dlsym(lib, "ncclCommInitRank"));
        allReduce = reinterpret_cast<decltype(allReduce)>(dlsym(lib, "ncclAllReduce"));
        commDestroy = reinterpret_cast<decltype(commDestroy)>(dlsym(lib, "ncclCommDestroy"));
        allGather = reinterpret_cast<decltype(allGather)>(dlsym(lib, "ncclAllGather"));
        send = reinterpret_cast<decltype(send)>(dlsym(lib, "ncclSend"));
        recv = reinterpret_cast<decltype(recv)>(dlsym(lib, "ncclRecv"));
        groupStart = reinterpret_cast<decltype(groupStart)>(dlsym(lib, "ncclGroupStart"));
        groupEnd = reinterpret_cast<decltype(groupEnd)>(dlsym(lib, "ncclGroupEnd"));
        commAbort = reinterpret_cast<decltype(commAbort)>(dlsym(lib, "ncclCommAbort"));
        commGetAsyncError = reinterpret_cast<decltype(commGetAsyncError)>(dlsym(lib, "ncclCommGetAsyncError"));
        if (!getUniqueId || !commInitRank || !allReduce || !commDestroy || !allGather || !send || !recv ||
            !groupStart || !groupEnd)
            return false;
        h = lib;
        return true;
    }
};
NcclApi nccl;

Ctx g;
std::mutex g_mu;

// A host wait with a deadline.  query(): 0 done, 1 pending, < 0 failed;
// async_error(): true when the communicator reports an error of its own;
// abort_comm(): called once when the wait gives up.  A peer that never joins a
// collective would otherwise keep the caller waiting for good: after timeout_ms
// (or on an asynchronous communicator error) the communicator is aborted, which
// makes its kernels return, and -9 comes back.
template <class Q, class AE, class AB>
int watch_wait(Q query, AE async_error, AB abort_comm, int timeout_ms) {
    const auto t0 = std::chrono::steady_clock::now();
    for (uint64_t it = 0;; ++it) {
        const int q = query();
        if (q == 0) return CZ_OK;
        if (q < 0) return CZ_ED2H;
        const auto us =
            std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count();
        if (async_error() || us >= (int64_t)timeout_ms * 1000) {
            abort_comm();
            return CZ_ENCCL;
        }
        // spin through the first 2 ms (decode calls end within it), then back off
        if (it >= 64 && us >= 2000) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

// Abort the EP communicator (caller holds g_mu): its kernels return, later EP
// calls return -9 until colizig_cuda_ep_shutdown + colizig_cuda_ep_init.
void ep_abort_locked() {
    if (g.ep_comm) {
        if (nccl.commAbort) nccl.commAbort(g.ep_comm);
        g.ep_comm = nullptr;
    }
    if (g.ep_on && g.ep_world > 1) g.ep_aborted = true;
}

// Synchronise `st`; watched (watch_wait) while an EP communicator is active.
int stream_sync(cudaStream_t st) {
    if (!g.ep_comm || g.ep_timeout_ms <= 0) return cudaStreamSynchronize(st) == cudaSuccess ? CZ_OK : CZ_ED2H;
    return watch_wait(
        [&]() -> int {
            const cudaError_t e = cudaStreamQuery(st);
            if (e == cudaSuccess) return 0;
            if (e == cudaErrorNotReady) return 1;
            return -1;
        },
        [&]() -> bool {
            ncclResult_t r = ncclSuccess;
            if (!nccl.commGetAsyncError || nccl.commGetAsyncError(g.ep_comm, &r) != ncclSuccess) return false;
            return r != ncclSuccess && r != ncclInProgress;
        },
        [&]() { ep_abort_locked(); }, g.ep_timeout_ms);
}

// Releases the in-kernel combine's buffers.  With `barrier`, first waits until
// every rank has reached this point with its kernels done (one NCCL all-reduce),
// so no peer still stores into the buffer freed here.
void ep_p2p_teardown_locked(bool barrier) {
    if (!g.ep_recv) return;
    cudaDeviceSynchronize();
    if (barrier && g.ep_comm) {
        DevBuf one;
        if (one.ensure(4) && cudaMemsetAsync(one.p, 0, 4, g.stream) == cudaSuccess &&
            nccl.allReduce(one.p, one.p, 1, ncclInt32, ncclSum, g.ep_comm, g.stream) == ncclSuccess)
            stream_sync(g.stream);
        cudaStreamSynchronize(g.stream);
        one.release();
    }
    for (int q = 0; q < cz::kEpMaxRanks; ++q) {
        if (g.ep_peer_map[q]) cudaIpcCloseMemHandle(g.ep_peer_map[q]);
        g.ep_peer_map[q] = nullptr;
        g.ep_slots[q] = nullptr;
    }
    cudaFree(g.ep_recv);
    g.ep_recv = nullptr;
    g.ep_p2p = false;
}

// Sets up the decode kernel's in-kernel combine (expert parallelism with
// replicated tokens): every rank allocates a zeroed receive buffer, the CUDA IPC
// handles go round with one NCCL all-gather, every rank maps its peers' buffers,
// and one NCCL all-reduce (min) of the outcomes decides for all ranks together.
// Any failure leaves the NCCL all-reduce combine in place.  Every rank takes
// part in both collectives whatever happened before them.
void ep_p2p_setup_locked() {
    const int W = g.ep_world, me = g.ep_rank;
    if (W < 2 || W > cz::kEpMaxRanks || !g.ep_comm) return;
    struct alignas(16) Rec {
        int ok;
        int pad;
        cudaIpcMemHandle_t h;
        char tail[128 - 8 - sizeof(cudaIpcMemHandle_t)];
    };
    static_assert(sizeof(Rec) == 128, "record size");
    Rec mine{};
    bool ok = cudaMalloc(&g.ep_recv, cz::kEpRecvBytes) == cudaSuccess;
    if (!ok) g.ep_recv = nullptr;
    ok = ok && cudaMemset(g.ep_recv, 0, cz::kEpRecvBytes) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
    ok = ok && cudaIpcGetMemHandle(&mine.h, g.ep_recv) == cudaSuccess;
    mine.ok = ok ? 1 : 0;
    std::vector<Rec> all(W);
    DevBuf rec, flag;
    bool coll = rec.ensure(sizeof(Rec) * W) && flag.ensure(4) &&
                cudaMemcpy(rec.as<uint8_t>() + sizeof(Rec) * me, &mine, sizeof(Rec), cudaMemcpyHostToDevice) ==
                    cudaSuccess;
    // the all-gather runs even after a local failure (the record says ok = 0)
    if (!coll || nccl.allGather(rec.as<uint8_t>() + sizeof(Rec) * me, rec.p, sizeof(Rec), ncclUint8, g.ep_comm,
                                g.stream) != ncclSuccess || stream_sync(g.stream) != CZ_OK ||
        cudaMemcpy(all.data(), rec.p, sizeof(Rec) * W, cudaMemcpyDeviceToHost) != cudaSuccess) {
        ok = false;
    }
    for (int q = 0; q < W && ok; ++q) ok = all[q].ok == 1;
    for (int q = 0; q < W && ok; ++q) {
        if (q == me) {
            g.ep_slots[q] = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(g.ep_recv) + cz::kEpRecvHeader);
            continue;
        }
        void* m = nullptr;
        if (cudaIpcOpenMemHandle(&m, all[q].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = false;
            break;
        }
        g.ep_peer_map[q] = m;
        g.ep_slots[q] = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(m) + cz::kEpRecvHeader);
    }
    int v = ok ? 1 : 0;
    bool agreed = flag.p && cudaMemcpy(flag.p, &v, 4, cudaMemcpyHostToDevice) == cudaSuccess &&
                  nccl.allReduce(flag.p, flag.p, 1, ncclInt32, ncclMin, g.ep_comm, g.stream) == ncclSuccess &&
                  stream_sync(g.stream) == CZ_OK && cudaMemcpy(&v, flag.p, 4, cudaMemcpyDeviceToHost) == cudaSuccess;
    rec.release();
    flag.release();
    if (agreed && v == 1) {
        g.ep_p2p = true;
        return;
    }
    ep_p2p_teardown_locked(false);
    cudaGetLastError();
}

// Forgets the cached device addresses of the no-allocation scratch (defined with
// colizig_cuda_moe_forward_noalloc below), so the first call after an init does
// the look-up again: a context reset by the host application reloads the module.
void noalloc_forget();

size_t nb(size_t x) { return (x + 127) / 128; }

// Token batches of at least this size take the prefill path (grouped GEMMs on
// tcgen05); smaller ones the decode kernel.
constexpr int kPrefillMinTokens = 32;

// Largest host-pointer transfer staged through the library's page-locked
// buffers (decode-sized calls); larger ones copy straight to/from the caller.
constexpr size_t kHostStageCap = 4u << 20;

int ensure_sync() {
    if (g.sync) return CZ_OK;
    if (cudaMalloc(&g.sync, cz::kSyncWords * sizeof(uint32_t)) != cudaSuccess) {
        g.sync = nullptr;
        return CZ_EALLOC;
    }
    if (cudaMemset(g.sync, 0, cz::kSyncWords * sizeof(uint32_t)) != cudaSuccess) return CZ_EALLOC;
    return CZ_OK;
}

void drop_host_graphs(bool all, uint32_t layer) {
    for (auto it = g.host_graphs.begin(); it != g.host_graphs.end();) {
        if (all || it->first.layer == layer) {
            cudaGraphExecDestroy(it->second);
            it = g.host_graphs.erase(it);
        } else {
            ++it;
        }
    }
    for (auto it = g.host_seen.begin(); it != g.host_seen.end();)
        it = (all || it->first.layer == layer) ? g.host_seen.erase(it) : std::next(it);
}

void free_layer(MoeLayer& L) {
    if (L.mem) cudaFree(L.mem);
    if (L.shb_mem) cudaFree(L.shb_mem);
    L = MoeLayer{};
}

void evict_lru_one() {
    if (g.lru.empty()) return;
    const uint64_t k = g.lru.back();
    g.lru.pop_back();
    auto it = g.keyed.find(k);
    if (it != g.keyed.end()) {
        cudaFree(it->second.w);
        cudaFree(it->second.s);
        g.used -= it->second.wb + it->second.sb;
        g.keyed.erase(it);
    }
}

void shutdown_locked() {
    if (!g.inited) return;
    cudaSetDevice(g.dev);
    cudaDeviceSynchronize();
    ep_p2p_teardown_locked(false);
    if (g.ep_comm) nccl.commDestroy(g.ep_comm);
    g.ep_comm = nullptr;
    g.ep_on = false;
    g.ep_rank = 0;
    g.ep_world = 1;
    for (auto& kv : g.keyed) {
        cudaFree(kv.second.w);
        cudaFree(kv.second.s);
    }
    g.keyed.clear();
    g.lru.clear();
    for (auto& kv : g.layers) free_layer(kv.second);
    g.layers.clear();
    drop_host_graphs(true, 0);
    g.io_host.release();
    g.io_xh.release();
    g.mm_xh.release();
    g.mm_yh.release();
    for (DevBuf* b : {&g.d_x, &g.d_y, &g.d_w, &g.d_s, &g.logits, &g.hrows, &g.pf_scratch, &g.shb_scratch, &g.io_x, &g.io_out, &g.io_res,
                      &g.ones, &g.sh_idx, &g.sh_gates, &g.sh_xn, &g.sh_slot, &g.sh_counts, &g.sh_allc,
                      &g.sh_tmp, &g.sh_send, &g.sh_recv, &g.sh_x, &g.sh_ridx, &g.sh_rgates, &g.sh_part, &g.sh_back})
        b->release();
    if (g.sync) cudaFree(g.sync);
    for (cudaEvent_t e : g.tm_ev) cudaEventDestroy(e);
    if (g.stream) cudaStreamDestroy(g.stream);
    g = Ctx{};
    noalloc_forget();
}

int init_locked(int device) {
    if (g.inited) return g.dev == device ? CZ_OK : -2;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n < 1) return -1;
    if (device < 0 || device >= n) return -2;
    if (cudaSetDevice(device) != cudaSuccess) return -2;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return -3;
    snprintf(g.name, sizeof g.name, "%s (sm_%d%d, %zu MiB)", prop.name, prop.major, prop.minor,
             (size_t)(prop.totalGlobalMem >> 20));
    g.num_sms = prop.multiProcessorCount;
    g.dev = device;
    if (cudaStreamCreateWithFlags(&g.stream, cudaStreamNonBlocking) != cudaSuccess) return -4;
    g.budget = 0;  // keyed store disabled until set (colizig_cuda.cu:184)
    g.inited = true;
    return CZ_OK;
}

// Copy `count` items of `bytes` each from per-expert source pointers into a
// contiguous destination, merging runs that are contiguous in the source.
template <class T>
int gather_copy(uint8_t* dst, const colizig_moe_expert* ex, int count, size_t bytes, T colizig_moe_expert::*field,
                cudaMemcpyKind kind) {
    int e = 0;
    while (e < count) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(ex[e].*field);
        if (!src) return CZ_EARGS;
        int run = 1;
        while (e + run < count && reinterpret_cast<const uint8_t*>(ex[e + run].*field) == src + run * bytes) ++run;
        if (cudaMemcpyAsync(dst + (size_t)e * bytes, src, (size_t)run * bytes, kind, g.stream) != cudaSuccess)
            return CZ_EH2D;
        e += run;
    }
    return CZ_OK;
}


// Like gather_copy for block-scale tables: every item is `rows` rows of
// `row_bytes`, written with a padded destination pitch (rows of the resident
// tables start on 16-byte boundaries, so kernels can bulk-copy them).
template <class T>
int gather_copy_2d(uint8_t* dst, size_t dst_pitch, const colizig_moe_expert* ex, int count, size_t rows,
                   size_t row_bytes, T colizig_moe_expert::*field, cudaMemcpyKind kind) {
    const size_t item = rows * row_bytes;
    int e = 0;
    while (e < count) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(ex[e].*field);
        if (!src) return CZ_EARGS;
        int run = 1;
        while (e + run < count && reinterpret_cast<const uint8_t*>(ex[e + run].*field) == src + run * item) ++run;
        if (cudaMemcpy2DAsync(dst + (size_t)e * rows * dst_pitch, dst_pitch, src, row_bytes, row_bytes,
                              (size_t)run * rows, kind, g.stream) != cudaSuccess)
            return CZ_EH2D;
        e += run;
    }
    return CZ_OK;
}

// A device buffer of at least `need` bytes whose new contents are zero: the
// decode kernel's tagged exchange words must not start with a stale tag.  Only
// a (re)allocation clears, and waits for the clear, so the steady state costs
// nothing.
bool ensure_zeroed(DevBuf& b, size_t need) {
    if (b.cap >= need && b.p) return true;
    if (!b.ensure(need)) return false;
    return cudaMemset(b.p, 0, b.cap) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
}

int ensure_decode_scratch(const colizig_moe_dims& d) {
    if (!ensure_zeroed(g.logits, cz::decode_logit_words((int)d.experts) * 8)) return CZ_EALLOC;
    if (!ensure_zeroed(g.hrows, cz::decode_hrow_words((int)d.topk, (int)d.inter, (int)d.shared_inter) * 8))
        return CZ_EALLOC;
    return ensure_sync();
}

cz::DecodeParams make_params(const MoeLayer& L) {
    cz::DecodeParams p{};
    p.router = L.router;
    p.gate_w = L.gate_w;
    p.up_w = L.up_w;
    p.down_w = L.down_w;
    p.gate_s = L.gate_s;
    p.up_s = L.up_s;
    p.down_s = L.down_s;
    p.sh_gate_w = L.sh_gate_w;
    p.sh_up_w = L.sh_up_w;
    p.sh_down_w = L.sh_down_w;
    p.sh_gate_s = L.sh_gate_s;
    p.sh_up_s = L.sh_up_s;
    p.sh_down_s = L.sh_down_s;
    p.sh_gate = L.sh_gate;
    p.H = (int)L.d.hidden;
    p.E = (int)L.d.experts;
    p.K = (int)L.d.topk;
    p.I = (int)L.d.inter;
    p.SI = (int)L.d.shared_inter;
    p.norm_topk = (int)L.d.norm_topk;
    p.e_lo = L.e_lo;
    p.e_hi = L.e_hi;
    p.shared_here = L.shared_here;
    p.gate_map = L.gate_map;
    p.up_map = L.up_map;
    p.sh_gate_map = L.shared_here ? L.sh_gate_map : L.gate_map;
    p.sh_up_map = L.shared_here ? L.sh_up_map : L.up_map;
    p.gu3d = L.gu_kb > 0;
    p.gu_kb = L.gu_kb;
    p.logits = g.logits.as<unsigned long long>();
    p.hrows = g.hrows.as<unsigned long long>();

    p.sync = g.sync;
    return p;
}

// Hands an armed failure-path hold (colizig_cuda_debug_hold_router) to this
// launch and disarms it: it applies to exactly one decode launch.
void take_debug_hold(cz::DecodeParams& p) {
    p.dbg_hold = g.dbg_hold;
    p.spin_limit = g.dbg_hold ? g.dbg_spin_limit : 0u;
    g.dbg_hold = 0;
    g.dbg_spin_limit = 0;
}

// Kernel timer.  Kinds of the recorded launch pairs.
constexpr int kTimerDecode = 1, kTimerPrefillGateUp = 2, kTimerPrefillDown = 3, kTimerMatmul = 4;

// Reserves `pairs` consecutive begin/end event pairs of the timer (all of kind
// `kind`); nullptr when the timer is off or full.  The events are recorded with
// cudaEventRecordExternal, so a forward captured into a CUDA graph keeps them as
// event-record nodes and every replay re-times the same launches.
cudaEvent_t* timer_take(int kind, int pairs) {
    if (g.tm_ev.empty()) return nullptr;
    if ((size_t)(g.tm_n + pairs) * 2 > g.tm_ev.size()) {
        g.tm_overflow = true;
        return nullptr;
    }
    cudaEvent_t* ev = g.tm_ev.data() + (size_t)g.tm_n * 2;
    for (int i = 0; i < pairs; ++i) g.tm_kind[g.tm_n++] = kind;
    return ev;
}

void timer_free() {
    for (cudaEvent_t e : g.tm_ev) cudaEventDestroy(e);
    g.tm_ev.clear();
    g.tm_kind.clear();
    g.tm_n = 0;
    g.tm_overflow = false;
}

// Runs one layer over T tokens (device pointers, stream-ordered), in launches
// of at most kDecodeMaxTokens tokens.
int moe_run_routed(const MoeLayer& L, const void* x, int x_bf16, int T, float* out, uint32_t* idx, float* gates,
                   const float* rms_w, float eps, const float* residual, cudaStream_t st, uint32_t* status_out) {
    if (T >= kPrefillMinTokens && L.pf_ok) {
        const size_t need = cz::prefill_scratch_bytes(T, (int)L.d.hidden, (int)L.d.experts, (int)L.d.topk,
                                                      (int)L.d.inter, (int)L.d.shared_inter, g.num_sms);
        if (!g.pf_scratch.ensure(need)) return CZ_EALLOC;
        if (ensure_sync()) return CZ_EALLOC;
        const float* res = residual && (!L.ep || g.ep_rank == 0) ? residual : nullptr;
        cudaEvent_t* ev = timer_take(kTimerPrefillGateUp, 2);
        if (ev) g.tm_kind[g.tm_n - 1] = kTimerPrefillDown;
        int rc = cz::prefill_run(L.pf, x, x_bf16, T, rms_w, eps, res, out, idx, gates, g.pf_scratch.p,
                                 g.pf_scratch.cap, g.sync + 1, g.num_sms, st, ev);
        if (rc) return rc;
        if (L.ep && g.ep_world > 1) {
            if (!g.ep_comm) return CZ_ENCCL;
            if (nccl.allReduce(out, out, (size_t)T * L.d.hidden, ncclFloat, ncclSum, g.ep_comm, st) != ncclSuccess)
                return CZ_ENCCL;
        }
        return CZ_OK;
    }
    int rc = ensure_decode_scratch(L.d);
    if (rc) return rc;
    const size_t xelt = x_bf16 ? 2 : 4;
    const int tmax = cz::decode_max_tokens((int)L.d.hidden, (int)L.d.experts, (int)L.d.topk, (int)L.d.inter,
                                           (int)L.d.shared_inter, x_bf16, g.num_sms);
    if (tmax < 1) return CZ_ESHAPE;
    // expert parallelism: the ranks' outputs are summed inside the decode kernel
    // (peer stores) when every rank mapped its peers' receive buffers, else by one
    // NCCL all-reduce after the launches; the choice is the same on every rank
    const bool ep_multi = L.ep && g.ep_world > 1;
    if (ep_multi && !g.ep_comm) return CZ_ENCCL;
    const bool p2p = ep_multi && g.ep_p2p && g.ep_p2p_use && L.d.hidden <= (uint32_t)cz::kEpMaxHidden &&
                     tmax <= cz::kDecodeMaxTokens;
    for (int t0 = 0; t0 < T; t0 += tmax) {
        const int n = T - t0 < tmax ? T - t0 : tmax;
        cz::DecodeParams p = make_params(L);
        if (p2p) {
            p.ep_world = g.ep_world;
            p.ep_rank = g.ep_rank;
            for (int q = 0; q < g.ep_world; ++q) p.ep_recv[q] = g.ep_slots[q];
            p.ep_seq = static_cast<uint32_t*>(g.ep_recv);
            // the peers' rows are waited for as long as the host waits for a collective
            p.ep_wait_ns = (uint64_t)(g.ep_timeout_ms > 0 ? g.ep_timeout_ms : 60000) * 1000000ull;
        }
        p.x = reinterpret_cast<const uint8_t*>(x) + (size_t)t0 * L.d.hidden * xelt;
        p.x_bf16 = x_bf16;
        p.T = n;
        p.rms_w = rms_w;
        p.eps = eps;
        // under expert parallelism the residual is added on rank 0 only (the all-reduce sums the ranks)
        p.residual = residual && (!L.ep || g.ep_rank == 0) ? residual + (size_t)t0 * L.d.hidden : nullptr;
        p.out = out + (size_t)t0 * L.d.hidden;
        p.topk_idx = idx ? idx + (size_t)t0 * L.d.topk : nullptr;
        p.topk_gates = gates ? gates + (size_t)t0 * L.d.topk : nullptr;
        p.status_out = t0 + n >= T ? status_out : nullptr;  // the last launch reports the error word
        cudaEvent_t* ev = timer_take(kTimerDecode, 1);
        if (ev && !cz::record_timer_event(ev[0], st)) return CZ_ELAUNCH;
        take_debug_hold(p);
        rc = cz::decode_launch(p, g.num_sms, st);
        if (rc) return rc;
        if (ev && !cz::record_timer_event(ev[1], st)) return CZ_ELAUNCH;
    }
    if (ep_multi && !p2p &&
        nccl.allReduce(out, out, (size_t)T * L.d.hidden, ncclFloat, ncclSum, g.ep_comm, st) != ncclSuccess)
        return CZ_ENCCL;
    return CZ_OK;
}

// One layer over T tokens: the routed experts (moe_run_routed) and, for a layer
// with a BF16 shared expert, its gate/up rows and sigmoid gate before them (from
// the layer input, which stack mode overwrites in place) and its down rows added
// into out after them (after the ranks' combine, so every rank's out has it).
int moe_run(const MoeLayer& L, const void* x, int x_bf16, int T, float* out, uint32_t* idx, float* gates,
            const float* rms_w, float eps, const float* residual, cudaStream_t st, uint32_t* status_out = nullptr) {
    if (!L.shb_si || T <= 0) return moe_run_routed(L, x, x_bf16, T, out, idx, gates, rms_w, eps, residual, st, status_out);
    const void* before = g.shb_scratch.p;
    if (!g.shb_scratch.ensure(cz::shb_scratch_bytes(T, (int)L.shb_si))) return CZ_EALLOC;
    if (before && before != g.shb_scratch.p) drop_host_graphs(true, 0);  // captured calls used the old scratch
    cz::ShbParams sp{};
    sp.x = x;
    sp.x_bf16 = x_bf16;
    sp.T = T;
    sp.H = (int)L.d.hidden;
    sp.SI = (int)L.shb_si;
    sp.rms_w = rms_w;
    sp.eps = eps;
    sp.wg = L.shb_g;
    sp.wu = L.shb_u;
    sp.wd = L.shb_d;
    sp.sh_gate = L.shb_gate;
    sp.hsh = g.shb_scratch.as<float>();
    sp.sg = reinterpret_cast<float*>(g.shb_scratch.as<uint8_t>() + ((size_t)T * L.shb_si * 4 + 255) / 256 * 256);
    sp.out = out;
    int rc = cz::shb_launch(sp, true, st);
    if (!rc) rc = moe_run_routed(L, x, x_bf16, T, out, idx, gates, rms_w, eps, residual, st, status_out);
    if (!rc) rc = cz::shb_launch(sp, false, st);
    return rc;
}

// Expert parallelism with sharded tokens (prefill): every rank passes its own
// T tokens (T may differ between ranks, 0 included) and gets their outputs.
// Each rank routes its tokens, sends every token row once to each rank holding
// one of its top-k experts (row + the token's ids and gates), runs the grouped
// pipeline on the rows it receives (pairs of experts held elsewhere are
// skipped), returns each row's partial sum, and adds its tokens' partials in
// ascending rank order (+ residual).  The exchanges are NCCL send/recv groups
// sized from one all-gather of the per-destination row counts (the host reads
// the counts, so this path synchronises the stream once per call).
int moe_run_sharded(const MoeLayer& L, const void* x, int x_bf16, int T, float* out, uint32_t* idx_out,
                    float* gates_out, const float* rms_w, float eps, const float* residual, cudaStream_t st) {
    if (!L.ep || g.ep_world < 2) return CZ_EARGS;
    if (!g.ep_comm) return CZ_ENCCL;  // aborted
    if (L.d.shared_inter || L.shb_si || !L.pf_ok) return CZ_ESHAPE;  // the same verdict on every rank (same layer)
    const int W = g.ep_world, me = g.ep_rank;
    const int K = (int)L.d.topk, E = (int)L.d.experts, H = (int)L.d.hidden;
    // Until the first collective, a failure here is only recorded: the rank still takes
    // part in the all-gather below (flagging itself), so its peers never wait for it.
    int local_rc = ensure_sync() ? CZ_EALLOC : CZ_OK;
    // 1. routing of this rank's tokens
    const size_t tk = (size_t)(T > 0 ? T : 1);
    if (!g.sh_idx.ensure(tk * K * 4) || !g.sh_gates.ensure(tk * K * 4) || !g.sh_slot.ensure(tk * W * 4) ||
        !g.sh_tmp.ensure(tk * 4) || (rms_w && !g.sh_xn.ensure(tk * H * 4)))
        local_rc = CZ_EALLOC;
    if (!g.sh_counts.ensure((size_t)(W + 5) * 4) || !g.sh_allc.ensure((size_t)W * (W + 5) * 4))
        return CZ_EALLOC;  // (a few bytes; without them there is nothing to exchange at all)
    if (!local_rc && T > 0) {
        const size_t need = cz::prefill_scratch_bytes(T, H, E, K, (int)L.d.inter, 0, g.num_sms);
        local_rc = g.pf_scratch.ensure(need)
                       ? cz::prefill_route(L.pf, x, x_bf16, T, rms_w, eps, g.sh_idx.as<uint32_t>(),
                                           g.sh_gates.as<float>(), rms_w ? g.sh_xn.as<float>() : nullptr,
                                           g.pf_scratch.p, g.pf_scratch.cap, st)
                       : CZ_EALLOC;
    }
    const void* xs = rms_w ? g.sh_xn.p : x;
    const int xbf = rms_w ? 0 : x_bf16;
    const size_t xrow = (size_t)H * (xbf ? 2 : 4);
    const size_t rs = (xrow + (size_t)8 * K + 15) & ~(size_t)15;
    // 2. destinations and row counts; 3. every rank's counts
    if (!local_rc)
        local_rc = cz::ep_plan(g.sh_idx.as<uint32_t>(), T, K, E, W, g.sh_slot.as<int>(), g.sh_counts.as<int>(),
                               g.sh_tmp.p, g.sh_tmp.cap, st);
    if (local_rc && cudaMemsetAsync(g.sh_counts.p, 0, (size_t)W * 4, st) != cudaSuccess) return local_rc;
    int rc = CZ_OK;
    // each rank's row: W counts, its row stride and its hidden size (so that every rank can
    // check that all of them will exchange rows of the same size), and the rows its current
    // buffers hold without allocating: receive side (exchange buffers, grouped-pipeline
    // scratch) and send side
    const auto rows_of = [](const DevBuf& b, size_t row) {
        return (int)std::min<size_t>(b.p ? b.cap / row : 0, (size_t)INT_MAX);
    };
    const int rbuf = std::min({rows_of(g.sh_recv, rs), rows_of(g.sh_x, xrow), rows_of(g.sh_ridx, (size_t)K * 4),
                               rows_of(g.sh_rgates, (size_t)K * 4), rows_of(g.sh_part, (size_t)H * 4)});
    int rpf = 0;  // largest R whose grouped-pipeline scratch fits (the size grows with R)
    for (int lo = 1, hi = rbuf; g.pf_scratch.p && lo <= hi;) {
        const int mid = lo + (hi - lo) / 2;
        if (cz::prefill_scratch_bytes(mid, H, E, K, (int)L.d.inter, 0, g.num_sms) <= g.pf_scratch.cap) {
            rpf = mid;
            lo = mid + 1;
        } else {
            hi = mid - 1;
        }
    }
    const int sbuf = std::min(rows_of(g.sh_send, rs), rows_of(g.sh_back, (size_t)H * 4));
    const int meta[5] = {local_rc ? -1 : (int)rs, H, rbuf, rpf, sbuf};  // rs -1: this rank failed, every rank stops
    if (cudaMemcpyAsync(g.sh_counts.as<int>() + W, meta, sizeof meta, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return CZ_EH2D;
    const int CW = W + 5;
    if (nccl.allGather(g.sh_counts.p, g.sh_allc.p, (size_t)CW, ncclInt32, g.ep_comm, st) != ncclSuccess) return CZ_ENCCL;
    std::vector<int> allc((size_t)W * CW);
    if (cudaMemcpyAsync(allc.data(), g.sh_allc.p, allc.size() * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return CZ_ED2H;
    if (const int src = stream_sync(st)) return src;
    for (int r = 0; r < W; ++r)  // the same verdict on every rank: no exchange of mismatched sizes
        if (allc[(size_t)r * CW + W] != (int)rs || allc[(size_t)r * CW + W + 1] != H)
            return local_rc ? local_rc : CZ_EARGS;
    std::vector<size_t> scnt(W), rcnt(W), soff(W + 1, 0), roff(W + 1, 0);
    for (int d = 0; d < W; ++d) {
        scnt[d] = (size_t)allc[(size_t)me * CW + d];
        rcnt[d] = (size_t)allc[(size_t)d * CW + me];
        soff[d + 1] = soff[d] + scnt[d];
        roff[d + 1] = roff[d] + rcnt[d];
    }
    const size_t S = soff[W], R = roff[W];
    // Does any rank have to allocate?  Every rank evaluates the same table, so all of them
    // take the same branch: without growth nothing below can fail and the exchange follows
    // directly; with growth every buffer is sized, then one all-reduce (min) of the ranks'
    // verdicts, so that no rank enters a send/recv its peers will not match.
    bool grow = false;
    for (int r = 0; r < W; ++r) {
        size_t Rr = 0, Sr = 0;
        for (int d = 0; d < W; ++d) {
            Rr += (size_t)allc[(size_t)d * CW + r];
            Sr += (size_t)allc[(size_t)r * CW + d];
        }
        const int* mr = &allc[(size_t)r * CW + W];
        grow |= std::max<size_t>(Rr, 1) > (size_t)mr[2] || (Rr > 0 && Rr > (size_t)mr[3]) ||
                std::max<size_t>(Sr, 1) > (size_t)mr[4];
    }
    const bool bufs_ok =
        g.sh_send.ensure_grow((S ? S : 1) * rs) && g.sh_recv.ensure_grow((R ? R : 1) * rs) &&
        g.sh_x.ensure_grow((R ? R : 1) * xrow) && g.sh_ridx.ensure_grow((R ? R : 1) * K * 4) &&
        g.sh_rgates.ensure_grow((R ? R : 1) * K * 4) && g.sh_part.ensure_grow((R ? R : 1) * (size_t)H * 4) &&
        g.sh_back.ensure_grow((S ? S : 1) * (size_t)H * 4) &&
        (R == 0 ||
         g.pf_scratch.ensure_grow(cz::prefill_scratch_bytes((int)R, H, E, K, (int)L.d.inter, 0, g.num_sms)));
    if (grow) {
        const int v = bufs_ok ? 1 : 0;
        int all = 0;
        int* dv = g.sh_tmp.as<int>();
        if (cudaMemcpyAsync(dv, &v, 4, cudaMemcpyHostToDevice, st) != cudaSuccess) return CZ_EH2D;
        if (nccl.allReduce(dv, dv, 1, ncclInt32, ncclMin, g.ep_comm, st) != ncclSuccess) return CZ_ENCCL;
        if (cudaMemcpyAsync(&all, dv, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) return CZ_ED2H;
        if (const int src = stream_sync(st)) return src;
        if (!all) return CZ_EALLOC;
    }
    // 4. pack; 5. exchange the rows
    rc = cz::ep_pack(xs, xrow, g.sh_idx.as<uint32_t>(), g.sh_gates.as<float>(), T, K, W, g.sh_slot.as<int>(),
                     g.sh_send.as<uint8_t>(), rs, st);
    if (rc) return rc;
    if (nccl.groupStart() != ncclSuccess) return CZ_ENCCL;
    for (int d = 0; d < W; ++d) {
        if (scnt[d] && nccl.send(g.sh_send.as<uint8_t>() + soff[d] * rs, scnt[d] * rs, ncclUint8, d, g.ep_comm, st) !=
                           ncclSuccess)
            rc = CZ_ENCCL;
        if (rcnt[d] && nccl.recv(g.sh_recv.as<uint8_t>() + roff[d] * rs, rcnt[d] * rs, ncclUint8, d, g.ep_comm, st) !=
                           ncclSuccess)
            rc = CZ_ENCCL;
    }
    if (nccl.groupEnd() != ncclSuccess || rc) return CZ_ENCCL;
    // 6. the experts held here over the received rows
    if (R) {
        rc = cz::ep_unpack(g.sh_recv.as<uint8_t>(), rs, (int)R, xrow, K, g.sh_x.p, g.sh_ridx.as<uint32_t>(),
                           g.sh_rgates.as<float>(), st);
        if (rc) return rc;
        cudaEvent_t* ev = timer_take(kTimerPrefillGateUp, 2);
        if (ev) g.tm_kind[g.tm_n - 1] = kTimerPrefillDown;
        rc = cz::prefill_run(L.pf, g.sh_x.p, xbf, (int)R, nullptr, 0.f, nullptr, g.sh_part.as<float>(), nullptr, nullptr,
                             g.pf_scratch.p, g.pf_scratch.cap, g.sync + 1, g.num_sms, st, ev, g.sh_ridx.as<uint32_t>(),
                             g.sh_rgates.as<float>());
        if (rc) return rc;
    }
    // 7. partial sums back to the rows' ranks
    if (nccl.groupStart() != ncclSuccess) return CZ_ENCCL;
    for (int d = 0; d < W; ++d) {
        if (rcnt[d] && nccl.send(g.sh_part.as<float>() + roff[d] * H, rcnt[d] * H, ncclFloat, d, g.ep_comm, st) !=
                           ncclSuccess)
            rc = CZ_ENCCL;
        if (scnt[d] && nccl.recv(g.sh_back.as<float>() + soff[d] * H, scnt[d] * H, ncclFloat, d, g.ep_comm, st) !=
                           ncclSuccess)
            rc = CZ_ENCCL;
    }
    if (nccl.groupEnd() != ncclSuccess || rc) return CZ_ENCCL;
    // 8. this rank's tokens: ranks in ascending order (+ residual)
    rc = cz::ep_combine(g.sh_back.as<float>(), g.sh_slot.as<int>(), T, W, H, residual, out, st);
    if (rc) return rc;
    if (T > 0 && idx_out &&
        cudaMemcpyAsync(idx_out, g.sh_idx.p, (size_t)T * K * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return CZ_ELAUNCH;
    if (T > 0 && gates_out &&
        cudaMemcpyAsync(gates_out, g.sh_gates.p, (size_t)T * K * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return CZ_ELAUNCH;
    return CZ_OK;
}

// Read and clear the device error word (synchronises `st`).
int check_device_error(cudaStream_t st) {
    if (!g.sync) return CZ_OK;
    uint32_t err = 0;
    if (cudaMemcpyAsync(&err, g.sync + 1, sizeof err, cudaMemcpyDeviceToHost, st) != cudaSuccess) return CZ_ED2H;
    if (const int src = stream_sync(st)) return src;
    if (err) {
        cudaMemsetAsync(g.sync + 1, 0, sizeof(uint32_t), st);
        cudaStreamSynchronize(st);
        return CZ_ETIMEOUT;
    }
    return CZ_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// ============================ Part 1 ============================

CZ_EXPORT int colizig_cuda_init(void) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    return init_locked(0);
}

// Same as colizig_cuda_init on an explicit device ordinal (one process per GPU
// for expert parallelism).  Not in the reference surface.
CZ_EXPORT int colizig_cuda_init_device(int device) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    return init_locked(device);
}

CZ_EXPORT const char* colizig_cuda_device_name(void) { return g.inited ? g.name : ""; }

// colizig_cuda_matmul_fp8's computation on device pointers, asynchronous on
// `stream` (NULL = the default stream): for hosts that keep activations and
// weights on the GPU (no keyed store, no staging).
CZ_EXPORT int colizig_cuda_matmul_fp8_device(float* y, const float* x, const unsigned char* w, const float* scales,
                                             int S, int I, int O, void* stream) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited || S < 1 || I < 1 || O < 1 || !y || !x || !w || !scales) return CZ_EARGS;
    cudaSetDevice(g.dev);
    return cz::fp8_matmul_launch(y, x, w, scales, S, I, O, reinterpret_cast<cudaStream_t>(stream));
}

CZ_EXPORT void colizig_cuda_set_vram_budget(uint64_t bytes) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return;
    cudaSetDevice(g.dev);
    size_t freeb = 0, totalb = 0;
    if (cudaMemGetInfo(&freeb, &totalb) == cudaSuccess) {
        const size_t cap = freeb - freeb / 8 + g.used;
        if (bytes > cap) bytes = cap;
    }
    g.budget = bytes;
    while (g.used > g.budget && !g.lru.empty()) evict_lru_one();
}

CZ_EXPORT void colizig_cuda_stats(uint64_t* hits, uint64_t* misses, uint64_t* uploaded_mib, uint64_t* resident) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (hits) *hits = g.hits;
    if (misses) *misses = g.misses;
    if (uploaded_mib) *uploaded_mib = g.uploaded >> 20;
    if (resident) *resident = (uint64_t)g.keyed.size();
}

CZ_EXPORT void colizig_cuda_shutdown(void) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    shutdown_locked();
}

CZ_EXPORT int colizig_cuda_matmul_fp8(float* y, const float* x, const unsigned char* w, const float* scales, int S,
                                      int I, int O, uint64_t key) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited || S < 1 || I < 1 || O < 1 || !y || !x || !w || !scales) return CZ_EARGS;
    cudaSetDevice(g.dev);
    const size_t xb = (size_t)S * I * sizeof(float);
    const size_t wb = (size_t)O * I;
    const size_t sb = nb(O) * nb(I) * sizeof(float);
    const size_t yb = (size_t)S * O * sizeof(float);
    if (!g.d_x.ensure(xb) || !g.d_y.ensure(yb)) return CZ_EALLOC;
    // decode-sized calls (the attention projections of one token, attn.zig:46-50) go through
    // the library's page-locked staging: x is copied from it, and the kernel writes y into
    // its mapped device view, so the call makes one host copy each way and no D2H copy
    const bool staged = xb <= kHostStageCap && yb <= kHostStageCap && g.mm_xh.ensure(xb) && g.mm_yh.ensure(yb);
    if (staged) memcpy(g.mm_xh.p, x, xb);
    if (cudaMemcpyAsync(g.d_x.p, staged ? g.mm_xh.p : x, xb, cudaMemcpyHostToDevice, g.stream) != cudaSuccess)
        return CZ_EH2D;

    const void* wdev = nullptr;
    const void* sdev = nullptr;
    if (key != 0 && g.budget != 0) {
        auto it = g.keyed.find(key);
        if (it != g.keyed.end() && it->second.wb == wb && it->second.sb == sb) {
            g.hits++;
            g.lru.splice(g.lru.begin(), g.lru, it->second.lru);
            wdev = it->second.w;
            sdev = it->second.s;
        } else {
            g.misses++;
            if (it != g.keyed.end()) {  // same key, new shape: drop the stale copy
                cudaFree(it->second.w);
                cudaFree(it->second.s);
                g.used -= it->second.wb + it->second.sb;
                g.lru.erase(it->second.lru);
                g.keyed.erase(it);
            }
            while (g.used + wb + sb > g.budget && !g.lru.empty()) evict_lru_one();
            Keyed k;
            if (g.used + wb + sb <= g.budget && cudaMalloc(&k.w, wb) == cudaSuccess) {
                if (cudaMalloc(&k.s, sb) != cudaSuccess) {
                    cudaFree(k.w);
                    k.w = nullptr;
                }
            } else {
                k.w = nullptr;
            }
            if (k.w) {
                if (cudaMemcpyAsync(k.w, w, wb, cudaMemcpyHostToDevice, g.stream) != cudaSuccess ||
                    cudaMemcpyAsync(k.s, scales, sb, cudaMemcpyHostToDevice, g.stream) != cudaSuccess) {
                    cudaFree(k.w);
                    cudaFree(k.s);
                    return CZ_EH2D;
                }
                k.wb = wb;
                k.sb = sb;
                g.lru.push_front(key);
                k.lru = g.lru.begin();
                g.keyed[key] = k;
                g.used += wb + sb;
                g.uploaded += wb + sb;
                wdev = k.w;
                sdev = k.s;
            }
        }
    }
    if (!wdev) {  // uncached (key 0, budget 0, or no room): upload into scratch
        if (!g.d_w.ensure(wb) || !g.d_s.ensure(sb)) return CZ_EALLOC;
        if (cudaMemcpyAsync(g.d_w.p, w, wb, cudaMemcpyHostToDevice, g.stream) != cudaSuccess) return CZ_EH2D;
        if (cudaMemcpyAsync(g.d_s.p, scales, sb, cudaMemcpyHostToDevice, g.stream) != cudaSuccess) return CZ_EH2D;
        g.uploaded += wb + sb;
        wdev = g.d_w.p;
        sdev = g.d_s.p;
    }
    float* const ydev = staged ? static_cast<float*>(g.mm_yh.dev) : g.d_y.as<float>();
    cudaEvent_t* ev = timer_take(kTimerMatmul, 1);
    if (ev && cudaEventRecord(ev[0], g.stream) != cudaSuccess) return CZ_ELAUNCH;
    if (cz::fp8_matmul_launch(ydev, g.d_x.as<float>(), (const uint8_t*)wdev, (const float*)sdev, S, I, O, g.stream) !=
        CZ_OK)
        return CZ_ELAUNCH;
    if (ev && cudaEventRecord(ev[1], g.stream) != cudaSuccess) return CZ_ELAUNCH;
    if (!staged && cudaMemcpyAsync(y, g.d_y.p, yb, cudaMemcpyDeviceToHost, g.stream) != cudaSuccess) return CZ_ED2H;
    if (cudaStreamSynchronize(g.stream) != cudaSuccess) return CZ_ED2H;
    if (staged) memcpy(y, g.mm_yh.p, yb);
    return CZ_OK;
}

// ============================ Part 2 ============================

CZ_EXPORT int colizig_cuda_moe_register_layer(uint32_t layer, const colizig_moe_dims* dims, const float* router,
                                              const colizig_moe_expert* experts, const colizig_moe_expert* shared,
                                              const float* shared_gate, uint32_t flags) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited || !dims || !router || !experts) return CZ_EARGS;
    colizig_moe_dims d = *dims;
    if (d.hidden == 0 || d.experts == 0 || d.topk == 0 || d.inter == 0 || d.topk > d.experts) return CZ_EARGS;
    if (d.topk > (uint32_t)cz::kMaxTopk || d.experts > (uint32_t)cz::kMaxExperts) return CZ_ESHAPE;
    if (d.hidden % 16 || d.inter % 16 || d.shared_inter % 16 || d.hidden > 16384 || d.inter > 32768 ||
        d.shared_inter > 32768)
        return CZ_ESHAPE;
    if (d.shared_inter && (!shared || !shared_gate)) return CZ_EARGS;
    // a BF16 shared expert is registered beside the routed experts, which then see none
    const uint32_t shb_si = (flags & COLIZIG_SHARED_BF16) ? d.shared_inter : 0u;
    if (shb_si) {
        if (!shared->gate_w || !shared->up_w || !shared->down_w) return CZ_EARGS;
        if (!cz::shb_supported((int)d.hidden, (int)shb_si)) return CZ_ESHAPE;
        d.shared_inter = 0;
    }
    const bool ep = (flags & COLIZIG_EP) != 0;
    if (ep && (!g.ep_on || (uint32_t)g.ep_world > d.experts)) return CZ_EARGS;
    cudaSetDevice(g.dev);
    const cudaMemcpyKind kind = (flags & COLIZIG_PTR_DEVICE) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    const size_t H = d.hidden, I = d.inter, SI = d.shared_inter;
    // expert parallelism: rank r holds the contiguous experts [r*E/W, (r+1)*E/W); rank 0
    // also holds the shared expert.  The router (and the shared gate vector) are replicated.
    const int e_lo = ep ? (int)((uint64_t)g.ep_rank * d.experts / g.ep_world) : 0;
    const int e_hi = ep ? (int)((uint64_t)(g.ep_rank + 1) * d.experts / g.ep_world) : (int)d.experts;
    const int shared_here = SI && (!ep || g.ep_rank == 0);
    const size_t ER = d.experts;          // router rows
    const size_t E = (size_t)(e_hi - e_lo);  // experts held here
    const size_t wexp = I * H;
    const size_t nbHp = (size_t)cz::cz_nbp((int)H), nbIp = (size_t)cz::cz_nbp((int)I), nbSIp = (size_t)cz::cz_nbp((int)SI);
    const size_t sexp = nb(I) * nbHp * 4, dexp = nb(H) * nbIp * 4;  // padded scale tables
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off = (off + bytes + 1023) & ~size_t(1023);  // 1024-aligned: swizzled TMA boxes need it
        return o;
    };
    const size_t o_router = take(ER * H * 4), o_gw = take(E * wexp), o_uw = take(E * wexp), o_dw = take(E * wexp);
    const size_t o_gs = take(E * sexp), o_us = take(E * sexp), o_ds = take(E * dexp);
    size_t o_shgw = 0, o_shuw = 0, o_shdw = 0, o_shgs = 0, o_shus = 0, o_shds = 0, o_shg = 0;
    if (shared_here) {
        o_shgw = take(SI * H);
        o_shuw = take(SI * H);
        o_shdw = take(SI * H);
        o_shgs = take(nb(SI) * nbHp * 4);
        o_shus = take(nb(SI) * nbHp * 4);
        o_shds = take(nb(H) * nbSIp * 4);
    }
    if (SI) o_shg = take(H * 4);
    MoeLayer L;
    L.d = d;
    L.bytes = off;
    L.e_lo = e_lo;
    L.e_hi = e_hi;
    L.shared_here = shared_here;
    L.ep = ep;
    if (cudaMalloc(&L.mem, off) != cudaSuccess) return CZ_EALLOC;
    uint8_t* base = reinterpret_cast<uint8_t*>(L.mem);
    L.router = reinterpret_cast<float*>(base + o_router);
    L.gate_w = base + o_gw;
    L.up_w = base + o_uw;
    L.down_w = base + o_dw;
    L.gate_s = reinterpret_cast<float*>(base + o_gs);
    L.up_s = reinterpret_cast<float*>(base + o_us);
    L.down_s = reinterpret_cast<float*>(base + o_ds);
    int rc = CZ_OK;
    if (cudaMemcpyAsync(L.router, router, ER * H * 4, kind, g.stream) != cudaSuccess) rc = CZ_EH2D;
    const int Ei = (int)E;
    experts += e_lo;
    if (!rc) rc = gather_copy(L.gate_w, experts, Ei, wexp, &colizig_moe_expert::gate_w, kind);
    if (!rc) rc = gather_copy(L.up_w, experts, Ei, wexp, &colizig_moe_expert::up_w, kind);
    if (!rc) rc = gather_copy(L.down_w, experts, Ei, wexp, &colizig_moe_expert::down_w, kind);
    if (!rc)
        rc = gather_copy_2d(reinterpret_cast<uint8_t*>(L.gate_s), nbHp * 4, experts, Ei, nb(I), nb(H) * 4,
                            &colizig_moe_expert::gate_s, kind);
    if (!rc)
        rc = gather_copy_2d(reinterpret_cast<uint8_t*>(L.up_s), nbHp * 4, experts, Ei, nb(I), nb(H) * 4,
                            &colizig_moe_expert::up_s, kind);
    if (!rc)
        rc = gather_copy_2d(reinterpret_cast<uint8_t*>(L.down_s), nbIp * 4, experts, Ei, nb(H), nb(I) * 4,
                            &colizig_moe_expert::down_s, kind);
    if (!rc && SI) {
        L.sh_gate = reinterpret_cast<float*>(base + o_shg);
        if (cudaMemcpyAsync(L.sh_gate, shared_gate, H * 4, kind, g.stream) != cudaSuccess) rc = CZ_EH2D;
    }
    if (!rc && shared_here) {
        L.sh_gate_w = base + o_shgw;
        L.sh_up_w = base + o_shuw;
        L.sh_down_w = base + o_shdw;
        L.sh_gate_s = reinterpret_cast<float*>(base + o_shgs);
        L.sh_up_s = reinterpret_cast<float*>(base + o_shus);
        L.sh_down_s = reinterpret_cast<float*>(base + o_shds);
        if (!shared->gate_w || !shared->up_w || !shared->down_w || !shared->gate_s || !shared->up_s ||
            !shared->down_s)
            rc = CZ_EARGS;
        const struct {
            void* dst;
            const void* src;
            size_t dpitch, rows, row_bytes;
        } cp[] = {{L.sh_gate_w, shared->gate_w, SI * H, 1, SI * H},
                  {L.sh_up_w, shared->up_w, SI * H, 1, SI * H},
                  {L.sh_down_w, shared->down_w, SI * H, 1, SI * H},
                  {L.sh_gate_s, shared->gate_s, nbHp * 4, nb(SI), nb(H) * 4},
                  {L.sh_up_s, shared->up_s, nbHp * 4, nb(SI), nb(H) * 4},
                  {L.sh_down_s, shared->down_s, nbSIp * 4, nb(H), nb(SI) * 4}};
        for (const auto& c : cp)
            if (!rc && cudaMemcpy2DAsync(c.dst, c.dpitch, c.src, c.row_bytes, c.row_bytes, c.rows, kind, g.stream) !=
                           cudaSuccess)
                rc = CZ_EH2D;
    }
    // decode tensor maps (gate/up); every map of a layer gets the same box depth
    if (!rc && E) {
        int kb = 0, kb2 = 0;
        if (!cz::make_gu_map(&L.gate_map, L.gate_w, E * I, H, &kb) || !cz::make_gu_map(&L.up_map, L.up_w, E * I, H, &kb2) ||
            kb != kb2)
            rc = CZ_ELAUNCH;
        L.gu_kb = kb;
    }
    if (!rc && shared_here) {
        int kb = 0, kb2 = 0;
        if (!cz::make_gu_map(&L.sh_gate_map, L.sh_gate_w, SI, H, &kb) ||
            !cz::make_gu_map(&L.sh_up_map, L.sh_up_w, SI, H, &kb2) || kb != kb2 || (E && kb != L.gu_kb))
            rc = CZ_ELAUNCH;
        L.gu_kb = kb;
    }
    if (!rc && E && cz::prefill_supported((int)H, (int)d.experts, (int)d.topk, (int)I, (int)SI)) {
        cz::PrefillLayer& P = L.pf;
        bool ok = cz::make_sw128_map(&P.gate_map, L.gate_w, E * I, H, 128) &&
                  cz::make_sw128_map(&P.up_map, L.up_w, E * I, H, 128) &&
                  cz::make_sw128_map(&P.down_map, L.down_w, E * H, I, 128);
        if (ok && shared_here)
            ok = cz::make_sw128_map(&P.sh_gate_map, L.sh_gate_w, SI, H, 128) &&
                 cz::make_sw128_map(&P.sh_up_map, L.sh_up_w, SI, H, 128) &&
                 cz::make_sw128_map(&P.sh_down_map, L.sh_down_w, H, SI, 128);
        P.router = L.router;
        P.sh_gate = L.sh_gate;
        P.gate_s = L.gate_s;
        P.up_s = L.up_s;
        P.down_s = L.down_s;
        P.sh_gate_s = L.sh_gate_s;
        P.sh_up_s = L.sh_up_s;
        P.sh_down_s = L.sh_down_s;
        P.H = (int)H;
        P.E = (int)d.experts;
        P.K = (int)d.topk;
        P.I = (int)I;
        P.SI = (int)SI;
        P.norm_topk = (int)d.norm_topk;
        P.e_lo = e_lo;
        P.e_hi = e_hi;
        P.shared_here = shared_here;
        L.pf_ok = ok;
    }
    if (!rc && shb_si) {
        // BF16 shared expert: gate, up [SI][H] and down [H][SI] bf16 bits, gate vector [H] f32
        const size_t wb = (size_t)shb_si * H * 2;
        const size_t o_g = 0, o_u = (wb + 255) & ~size_t(255), o_d = 2 * o_u, o_v = 3 * o_u;
        if (cudaMalloc(&L.shb_mem, o_v + H * 4) != cudaSuccess) {
            L.shb_mem = nullptr;
            rc = CZ_EALLOC;
        } else {
            uint8_t* b = static_cast<uint8_t*>(L.shb_mem);
            L.shb_si = shb_si;
            L.shb_g = reinterpret_cast<uint16_t*>(b + o_g);
            L.shb_u = reinterpret_cast<uint16_t*>(b + o_u);
            L.shb_d = reinterpret_cast<uint16_t*>(b + o_d);
            L.shb_gate = reinterpret_cast<float*>(b + o_v);
            if (cudaMemcpyAsync(L.shb_g, shared->gate_w, wb, kind, g.stream) != cudaSuccess ||
                cudaMemcpyAsync(L.shb_u, shared->up_w, wb, kind, g.stream) != cudaSuccess ||
                cudaMemcpyAsync(L.shb_d, shared->down_w, wb, kind, g.stream) != cudaSuccess ||
                cudaMemcpyAsync(L.shb_gate, shared_gate, H * 4, kind, g.stream) != cudaSuccess)
                rc = CZ_EH2D;
        }
    }
    if (!rc && cudaStreamSynchronize(g.stream) != cudaSuccess) rc = CZ_EH2D;
    if (rc) {
        cudaStreamSynchronize(g.stream);
        free_layer(L);
        return rc;
    }
    auto it = g.layers.find(layer);
    if (it != g.layers.end()) free_layer(it->second);
    drop_host_graphs(false, layer);
    L.serial = g.next_serial++;
    g.layers[layer] = L;
    return CZ_OK;
}

CZ_EXPORT int colizig_cuda_moe_unregister_layer(uint32_t layer) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g.layers.find(layer);
    if (it == g.layers.end()) return CZ_ENOLAYER;
    cudaSetDevice(g.dev);
    cudaDeviceSynchronize();
    drop_host_graphs(false, layer);
    free_layer(it->second);
    g.layers.erase(it);
    return CZ_OK;
}

CZ_EXPORT int colizig_cuda_moe_forward(uint32_t layer, const void* x, int x_dtype, int T, float* out,
                                       uint32_t* topk_idx, float* topk_gates, uint32_t flags, void* stream) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited || T < 0 || (T > 0 && (!x || !out)) || (x_dtype != COLIZIG_X_F32 && x_dtype != COLIZIG_X_BF16))
        return CZ_EARGS;
    auto it = g.layers.find(layer);
    if (it == g.layers.end()) return CZ_ENOLAYER;
    const bool sharded = flags & COLIZIG_EP_SHARDED;
    if (sharded && !it->second.ep) return CZ_EARGS;
    if (T == 0 && !sharded) return CZ_OK;  // a sharded call takes part in the exchange even without tokens
    cudaSetDevice(g.dev);
    const MoeLayer& L = it->second;
    const size_t H = L.d.hidden, K = L.d.topk;
    const int bf16 = x_dtype == COLIZIG_X_BF16;
    const size_t xb = (size_t)T * H * (bf16 ? 2 : 4), ob = (size_t)T * H * 4, kb = (size_t)T * K * 4;
    auto run = [&](const void* xd, float* od, uint32_t* id, float* gd, cudaStream_t st, uint32_t* status = nullptr) {
        return sharded ? moe_run_sharded(L, xd, bf16, T, od, id, gd, nullptr, 0.f, nullptr, st)
                       : moe_run(L, xd, bf16, T, od, id, gd, nullptr, 0.f, nullptr, st, status);
    };
    if (flags & COLIZIG_PTR_DEVICE) {
        if (T > 0 && (!aligned16(x) || !aligned16(out))) return CZ_EARGS;
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        return run(x, out, topk_idx, topk_gates, st);
    }
    // host pointers: synchronous on the library stream.  The results land in one
    // device buffer [out][top-k ids][top-k gates][error word] (256-byte aligned
    // parts) and come back in one copy through pinned staging, followed by one
    // stream synchronisation: a small copy costs mostly its fixed latency.  The
    // tokens go up through pinned staging too (a pageable source would make the
    // driver stage them itself).  Past kHostStageCap bytes (prefill batches) the
    // copies go straight between the caller's buffers and the device instead, so
    // the page-locked staging stays small.
    const auto up256 = [](size_t n) { return (n + 255) & ~(size_t)255; };
    const size_t io = up256(ob), go = io + (topk_idx ? up256(kb) : 0);
    const size_t eo = go + (topk_gates ? up256(kb) : 0);
    const size_t rb = eo + sizeof(uint32_t);
    const bool staged = rb <= kHostStageCap && xb <= kHostStageCap;
    if (!g.io_x.ensure(xb) || !g.io_res.ensure(rb) || (staged && (!g.io_host.ensure(rb) || !g.io_xh.ensure(xb))) ||
        ensure_sync())
        return CZ_EALLOC;
    uint8_t* const res = g.io_res.as<uint8_t>();
    // decode launches copy the error word into the result buffer themselves (their
    // last CTA); the other paths get one device-to-device copy of it below
    const bool kernel_status = staged && !sharded && !(T >= kPrefillMinTokens && L.pf_ok);
    // Decode-sized calls on a single GPU are replayed from a captured CUDA graph
    // (the token upload and the decode launches), one launch call per forward;
    // the kernel writes outputs, top-k and the error word straight into the mapped
    // pinned staging, so no copy back is needed.  A key's first call runs directly
    // (it allocates the decode scratch and sets the kernel attributes); the second
    // captures.
    // (expert-parallel layers too when the decode kernel sums the ranks itself: no
    // NCCL call is captured, and every rank replays the same launches)
    const bool ep_kernel_combine = L.ep && g.ep_world > 1 && g.ep_p2p && g.ep_p2p_use && g.ep_comm &&
                                   L.d.hidden <= (uint32_t)cz::kEpMaxHidden;
    const bool graphable = kernel_status && (!L.ep || ep_kernel_combine) && xb && ob && !g.dbg_hold &&
                           g.tm_ev.empty();
    if (graphable && ensure_decode_scratch(L.d) == CZ_OK) {
        const HostGraphKey key{layer, L.serial, T, bf16, topk_idx != nullptr, topk_gates != nullptr, g.io_x.p,
                               g.io_res.p, g.io_host.p, g.io_xh.p, g.logits.p, g.hrows.p, g.sync};
        auto gi = g.host_graphs.find(key);
        if (gi == g.host_graphs.end() && g.host_seen.count(key)) {
            if (g.host_graphs.size() >= 4096) drop_host_graphs(true, 0);
            cudaGraph_t graph = nullptr;
            cudaGraphExec_t exec = nullptr;
            bool ok = cudaStreamBeginCapture(g.stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
            if (ok) {
                ok = cudaMemcpyAsync(g.io_x.p, g.io_xh.p, xb, cudaMemcpyHostToDevice, g.stream) == cudaSuccess;
                uint8_t* const hd = static_cast<uint8_t*>(g.io_host.dev);
                ok = ok && moe_run(L, g.io_x.p, bf16, T, reinterpret_cast<float*>(hd),
                                   topk_idx ? reinterpret_cast<uint32_t*>(hd + io) : nullptr,
                                   topk_gates ? reinterpret_cast<float*>(hd + go) : nullptr, nullptr, 0.f, nullptr,
                                   g.stream, reinterpret_cast<uint32_t*>(hd + eo)) == CZ_OK;
                const bool ended = cudaStreamEndCapture(g.stream, &graph) == cudaSuccess;
                ok = ok && ended && cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
                if (graph) cudaGraphDestroy(graph);
            }
            if (ok) {
                gi = g.host_graphs.emplace(key, exec).first;
            } else {
                if (exec) cudaGraphExecDestroy(exec);
                cudaGetLastError();  // a failed capture leaves nothing behind: run directly
            }
        }
        if (gi != g.host_graphs.end()) {
            memcpy(g.io_xh.p, x, xb);
            if (cudaGraphLaunch(gi->second, g.stream) != cudaSuccess) return CZ_ELAUNCH;
            if (const int src = stream_sync(g.stream)) return src;
            const uint8_t* const hs = static_cast<const uint8_t*>(g.io_host.p);
            uint32_t err = 0;
            memcpy(&err, hs + eo, sizeof err);
            if (err) {
                cudaMemsetAsync(g.sync + 1, 0, sizeof(uint32_t), g.stream);
                cudaStreamSynchronize(g.stream);
                return CZ_ETIMEOUT;
            }
            memcpy(out, hs, ob);
            if (topk_idx) memcpy(topk_idx, hs + io, kb);
            if (topk_gates) memcpy(topk_gates, hs + go, kb);
            return CZ_OK;
        }
        if (g.host_seen.size() >= 8192) g.host_seen.clear();
        g.host_seen[key] = 1;
    }
    if (xb) {
        const void* src = x;
        if (staged) {
            memcpy(g.io_xh.p, x, xb);
            src = g.io_xh.p;
        }
        if (cudaMemcpyAsync(g.io_x.p, src, xb, cudaMemcpyHostToDevice, g.stream) != cudaSuccess) return CZ_EH2D;
    }
    int rc = run(g.io_x.p, reinterpret_cast<float*>(res), topk_idx ? reinterpret_cast<uint32_t*>(res + io) : nullptr,
                 topk_gates ? reinterpret_cast<float*>(res + go) : nullptr, g.stream,
                 kernel_status ? reinterpret_cast<uint32_t*>(res + eo) : nullptr);
    if (rc) {
        stream_sync(g.stream);
        return rc;
    }
    if (!ob) return check_device_error(g.stream);
    if (!staged) {
        if (cudaMemcpyAsync(out, res, ob, cudaMemcpyDeviceToHost, g.stream) != cudaSuccess ||
            (topk_idx && cudaMemcpyAsync(topk_idx, res + io, kb, cudaMemcpyDeviceToHost, g.stream) != cudaSuccess) ||
            (topk_gates && cudaMemcpyAsync(topk_gates, res + go, kb, cudaMemcpyDeviceToHost, g.stream) != cudaSuccess))
            return CZ_ED2H;
        return check_device_error(g.stream);  // synchronises the stream
    }
    if ((!kernel_status &&
         cudaMemcpyAsync(res + eo, g.sync + 1, sizeof(uint32_t), cudaMemcpyDeviceToDevice, g.stream) != cudaSuccess) ||
        cudaMemcpyAsync(g.io_host.p, res, rb, cudaMemcpyDeviceToHost, g.stream) != cudaSuccess)
        return CZ_ED2H;
    if (const int src = stream_sync(g.stream)) return src;
    const uint8_t* const hs = static_cast<const uint8_t*>(g.io_host.p);
    uint32_t err = 0;
    memcpy(&err, hs + eo, sizeof err);
    if (err) {
        cudaMemsetAsync(g.sync + 1, 0, sizeof(uint32_t), g.stream);
        cudaStreamSynchronize(g.stream);
        return CZ_ETIMEOUT;
    }
    memcpy(out, hs, ob);
    if (topk_idx) memcpy(topk_idx, hs + io, kb);
    if (topk_gates) memcpy(topk_gates, hs + go, kb);
    return CZ_OK;
}

CZ_EXPORT int colizig_cuda_moe_stack_forward(uint32_t first_layer, uint32_t n_layers, const float* norm_w, float eps,
                                             float* h, int T, uint32_t flags, void* stream) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited || !h || T < 0) return CZ_EARGS;
    const bool sharded = flags & COLIZIG_EP_SHARDED;
    if (n_layers == 0 || (T == 0 && !sharded)) return CZ_OK;  // sharded: every rank takes part in every layer
    std::vector<const MoeLayer*> Ls;
    for (uint32_t l = 0; l < n_layers; ++l) {
        auto it = g.layers.find(first_layer + l);
        if (it == g.layers.end()) return CZ_ENOLAYER;
        if (it->second.d.hidden != g.layers.find(first_layer)->second.d.hidden) return CZ_ESHAPE;
        Ls.push_back(&it->second);
    }
    cudaSetDevice(g.dev);
    const size_t H = Ls[0]->d.hidden;
    const bool dev = flags & COLIZIG_PTR_DEVICE;
    cudaStream_t st = dev ? reinterpret_cast<cudaStream_t>(stream) : g.stream;
    // norm weights: caller's (device or host) or all ones
    const float* nw = norm_w;
    if (!nw || !dev) {
        if (!g.ones.ensure((size_t)n_layers * H * 4)) return CZ_EALLOC;
        if (!nw) {
            std::vector<float> ones((size_t)n_layers * H, 1.0f);
            if (cudaMemcpyAsync(g.ones.p, ones.data(), ones.size() * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                cudaStreamSynchronize(st) != cudaSuccess)
                return CZ_EH2D;
        } else if (cudaMemcpyAsync(g.ones.p, nw, (size_t)n_layers * H * 4, cudaMemcpyHostToDevice, st) !=
                   cudaSuccess) {
            return CZ_EH2D;
        }
        nw = g.ones.as<float>();
    }
    float* hd = h;
    if (!dev) {
        if (!g.io_out.ensure((size_t)T * H * 4)) return CZ_EALLOC;
        if (cudaMemcpyAsync(g.io_out.p, h, (size_t)T * H * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
            return CZ_EH2D;
        hd = g.io_out.as<float>();
    } else if (!aligned16(h)) {
        return CZ_EARGS;
    }
    for (uint32_t l = 0; l < n_layers; ++l) {
        const int rc = sharded ? moe_run_sharded(*Ls[l], hd, 0, T, hd, nullptr, nullptr, nw + (size_t)l * H, eps, hd, st)
                               : moe_run(*Ls[l], hd, 0, T, hd, nullptr, nullptr, nw + (size_t)l * H, eps, hd, st);
        if (rc) {
            cudaStreamSynchronize(st);
            return rc;
        }
    }
    if (!dev) {
        if (cudaMemcpyAsync(h, hd, (size_t)T * H * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) return CZ_ED2H;
        return check_device_error(st);
    }
    return CZ_OK;
}

CZ_EXPORT int colizig_cuda_moe_check(void* stream) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return CZ_EARGS;
    cudaSetDevice(g.dev);
    // NULL is the default stream, as for the device-pointer forward: the read is
    // ordered after the calls issued there
    return check_device_error(reinterpret_cast<cudaStream_t>(stream));
}

// Kernel timer for benchmarks (not in the reference surface).  capacity > 0
// (re)arms it with room for `capacity` launch pairs and clears what it held;
// capacity 0 turns it off.  While armed, colizig_cuda_moe_forward* record a CUDA
// event pair around every decode kernel launch and around each of the two grouped
// GEMM launches of a prefill forward, so that the launches' own device time can be
// read back, also from inside a captured CUDA graph.
CZ_EXPORT int colizig_cuda_kernel_timer(int capacity) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return CZ_EARGS;
    if (capacity < 0 || capacity > (1 << 20)) return CZ_EARGS;
    cudaSetDevice(g.dev);
    timer_free();
    g.tm_ev.resize((size_t)capacity * 2, nullptr);
    g.tm_kind.assign((size_t)capacity, 0);
    for (cudaEvent_t& e : g.tm_ev)
        if (cudaEventCreate(&e) != cudaSuccess) {
            e = nullptr;
            timer_free();
            return CZ_EALLOC;
        }
    return CZ_OK;
}

// Reads the timer: for up to max_n recorded pairs, their kind (1 decode kernel,
// 2 prefill gate/up GEMM, 3 prefill down GEMM) and device time in ms.  Waits for
// the recorded events.  Returns the number of pairs written, or a negative
// result code (CZ_EALLOC when some pairs were dropped because the timer was full).
CZ_EXPORT int colizig_cuda_kernel_timer_read(int* kinds, float* ms, int max_n) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return CZ_EARGS;
    if (max_n < 0 || (max_n && (!kinds || !ms))) return CZ_EARGS;
    if (g.tm_overflow) return CZ_EALLOC;
    cudaSetDevice(g.dev);
    const int n = g.tm_n < max_n ? g.tm_n : max_n;
    for (int i = 0; i < n; ++i) {
        if (cudaEventSynchronize(g.tm_ev[2 * i + 1]) != cudaSuccess) return CZ_ED2H;
        float t = 0.f;
        if (cudaEventElapsedTime(&t, g.tm_ev[2 * i], g.tm_ev[2 * i + 1]) != cudaSuccess) return CZ_ED2H;
        kinds[i] = g.tm_kind[i];
        ms[i] = t;
    }
    return n;
}

// Failure-path test hook (no reference counterpart): the next decode launch
// withholds router row 0's logits, so every CTA's bounded wait for them gives up
// after `spin_limit` polls (about 0.2 us each) and the launch ends early with
// the error word set.  Nothing faults and nothing hangs.
CZ_EXPORT int colizig_cuda_debug_hold_router(uint32_t spin_limit) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited || spin_limit == 0) return CZ_EARGS;
    g.dbg_hold = 1;
    g.dbg_spin_limit = spin_limit;
    return CZ_OK;
}

// Diagnostics: the device error word's bits as they stand (after all device
// work so far has finished), without clearing them; 0 before any MoE call.
CZ_EXPORT int colizig_cuda_debug_error_bits(uint32_t* bits) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited || !bits) return CZ_EARGS;
    cudaSetDevice(g.dev);
    *bits = 0;
    if (!g.sync) return CZ_OK;
    if (cudaDeviceSynchronize() != cudaSuccess) return CZ_ED2H;
    return cudaMemcpy(bits, g.sync + 1, sizeof(uint32_t), cudaMemcpyDeviceToHost) == cudaSuccess ? CZ_OK : CZ_ED2H;
}

CZ_EXPORT int colizig_cuda_debug_expf(const float* x_dev, float* y_dev, size_t n) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited || (!x_dev && n) || (!y_dev && n)) return CZ_EARGS;
    cudaSetDevice(g.dev);
    int rc = cz::debug_expf_launch(x_dev, y_dev, n, g.stream);
    if (rc) return rc;
    return cudaStreamSynchronize(g.stream) == cudaSuccess ? CZ_OK : CZ_ELAUNCH;
}

// ---- expert parallelism --------------------------------------------------

CZ_EXPORT int colizig_cuda_ep_unique_id(void* id_out) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!id_out) return CZ_EARGS;
    if (!nccl.load()) return CZ_ENCCL;
    ncclUniqueId id;
    if (nccl.getUniqueId(&id) != ncclSuccess) return CZ_ENCCL;
    memcpy(id_out, &id, sizeof id);
    return CZ_OK;
}

CZ_EXPORT int colizig_cuda_ep_init(int rank, int world, const void* id) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited || world < 1 || rank < 0 || rank >= world || (world > 1 && !id)) return CZ_EARGS;
    if (g.ep_on) return CZ_EARGS;  // once per process (until colizig_cuda_ep_shutdown)
    cudaSetDevice(g.dev);
    if (world > 1) {
        if (!nccl.load()) return CZ_ENCCL;
        ncclUniqueId uid;
        memcpy(&uid, id, sizeof uid);
        ncclComm_t comm = nullptr;
        if (nccl.commInitRank(&comm, world, uid, rank) != ncclSuccess) return CZ_ENCCL;
        g.ep_comm = comm;
    }
    g.ep_rank = rank;
    g.ep_world = world;
    g.ep_on = true;
    ep_p2p_setup_locked();  // collective: every rank of the communicator is here too
    return CZ_OK;
}

CZ_EXPORT int colizig_cuda_ep_shutdown(void) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return CZ_OK;
    cudaSetDevice(g.dev);
    cudaDeviceSynchronize();
    for (auto& kv : g.layers)
        if (kv.second.ep) return CZ_EARGS;  // unregister the expert-parallel layers first
    ep_p2p_teardown_locked(true);
    if (g.ep_comm) nccl.commDestroy(g.ep_comm);
    g.ep_comm = nullptr;
    g.ep_on = false;
    g.ep_aborted = false;
    g.ep_rank = 0;
    g.ep_world = 1;
    return CZ_OK;
}

// Deadline of the library's host waits while an EP communicator is active
// (<= 0: unwatched); see watch_wait.
CZ_EXPORT int colizig_cuda_ep_set_timeout(int ms) {
    std::lock_guard<std::mutex> lk(g_mu);
    g.ep_timeout_ms = ms;
    drop_host_graphs(true, 0);  // captured decode launches carry the kernel's wait deadline
    return CZ_OK;
}

// Abort the EP communicator now (a host watchdog that learned a peer has left
// calls it between steps): its kernels return, and EP calls return -9 until
// colizig_cuda_ep_shutdown + colizig_cuda_ep_init.  Needs no device work.
CZ_EXPORT int colizig_cuda_ep_abort(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    ep_abort_locked();
    return CZ_OK;
}

// Tokens one decode launch of this layer takes (a decode-sized call of T tokens is
// ceil(T / n) launches); 0 when the layer is unknown or the decode kernel cannot
// take its dims.
CZ_EXPORT int colizig_cuda_moe_decode_batch(uint32_t layer, int x_dtype) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g.layers.find(layer);
    if (!g.inited || it == g.layers.end() || (x_dtype != COLIZIG_X_F32 && x_dtype != COLIZIG_X_BF16)) return 0;
    const colizig_moe_dims& d = it->second.d;
    return cz::decode_max_tokens((int)d.hidden, (int)d.experts, (int)d.topk, (int)d.inter, (int)d.shared_inter,
                                 x_dtype == COLIZIG_X_BF16, g.num_sms);
}

// How expert-parallel decode calls sum the ranks: 1 = inside the decode kernel
// (peer stores into every rank's receive buffer), 0 = one NCCL all-reduce per call.
CZ_EXPORT int colizig_cuda_ep_combine_mode(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    return g.ep_p2p && g.ep_p2p_use ? 1 : 0;
}

// Chooses the decode combine: 1 = inside the kernel when it was set up at
// colizig_cuda_ep_init (the default), 0 = NCCL all-reduce.  Every rank must make
// the same choice before its next EP call.
CZ_EXPORT int colizig_cuda_ep_set_combine(int in_kernel) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (in_kernel != 0 && in_kernel != 1) return CZ_EARGS;
    if (g.ep_p2p_use != (in_kernel == 1)) drop_host_graphs(true, 0);
    g.ep_p2p_use = in_kernel == 1;
    return CZ_OK;
}

// Test hook for the watched wait: watch_wait over caller-provided fakes of the
// stream query, the communicator's error report and the abort.
CZ_EXPORT int colizig_cuda_debug_watch_wait(int (*query)(void*), int (*async_error)(void*), void (*abort_comm)(void*),
                                            void* ctx, int timeout_ms) {
    if (!query || !async_error || !abort_comm) return CZ_EARGS;
    return watch_wait([&]() { return query(ctx); }, [&]() { return async_error(ctx) != 0; },
                      [&]() { abort_comm(ctx); }, timeout_ms);
}

// ---- colizig_cuda_moe_forward_noalloc -------------------------------------
// The device-pointer forward with its scratch in one static device array
// instead of cudaMalloc'd buffers: [sync words][router logits][h rows of every
// (token, expert) pair].  Static device storage is zero when the module loads,
// which is what the sync words and the tagged exchange words need (every launch
// zeroes the counter region the next launch uses, and tags the words it writes
// with its own sequence number, which a zero word never carries).
namespace {

constexpr int kNoAllocMaxHidden = 4096;
constexpr int kNoAllocMaxTokens = 4;  // tokens per launch through the static scratch
constexpr size_t kNoAllocSyncBytes = 768;
constexpr int kNoAllocMaxInter = 1024;  // moe_intermediate and shared_intermediate
// tagged 8-byte exchange words (router logits, h rows), as the decode kernel reads them
constexpr size_t kNoAllocLogitBytes = (size_t)kNoAllocMaxTokens * ((cz::kMaxExperts + 1 + 3) & ~3) * 8;
constexpr size_t kNoAllocHBytes = (size_t)kNoAllocMaxTokens * (cz::kMaxTopk + 1) * kNoAllocMaxInter * 8;
constexpr size_t kNoAllocBytes = kNoAllocSyncBytes + kNoAllocLogitBytes + kNoAllocHBytes;
static_assert(kNoAllocMaxTokens <= cz::kDecodeMaxTokens, "one launch's scratch");
static_assert(cz::kSyncWords * sizeof(uint32_t) <= kNoAllocSyncBytes, "sync words");
static_assert(kNoAllocBytes == 574336, "the size stated in colizig_cuda.h");

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

constexpr int kNoAllocMaxDevices = 64;
uint8_t* g_noalloc_addr[kNoAllocMaxDevices] = {};

void noalloc_forget() {
    for (int i = 0; i < kNoAllocMaxDevices; ++i) g_noalloc_addr[i] = nullptr;
}

// Address of the static scratch on device `dev`: looked up on the first call
// for that device after an init (set-up), cached until shutdown.
uint8_t* noalloc_scratch(int dev) {
    if (dev < 0 || dev >= kNoAllocMaxDevices) return nullptr;
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return nullptr;
        g_noalloc_addr[dev] = static_cast<uint8_t*>(p);
    }
    return g_noalloc_addr[dev];
}

}  // namespace

CZ_EXPORT int colizig_cuda_moe_forward_noalloc(uint32_t layer, const void* x, int x_dtype, int T, float* out,
                                               uint32_t* topk_idx, float* topk_gates, uint32_t* status,
                                               void* stream) {
    CsrGuard _csr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited || !x || !out || T < 0 || (x_dtype != COLIZIG_X_F32 && x_dtype != COLIZIG_X_BF16))
        return CZ_EARGS;
    auto it = g.layers.find(layer);
    if (it == g.layers.end()) return CZ_ENOLAYER;
    const MoeLayer& L = it->second;
    if (L.ep) return CZ_EARGS;  // its all-reduce is not part of this entry point
    if (L.shb_si) return CZ_ESHAPE;  // the BF16 shared expert's scratch is allocated
    if (L.d.hidden > (uint32_t)kNoAllocMaxHidden || L.d.experts > (uint32_t)cz::kMaxExperts ||
        L.d.topk > (uint32_t)cz::kMaxTopk || g.num_sms > cz::kMaxGrid ||
        L.d.inter > (uint32_t)kNoAllocMaxInter || L.d.shared_inter > (uint32_t)kNoAllocMaxInter)
        return CZ_ESHAPE;
    if (!aligned16(x) || !aligned16(out)) return CZ_EARGS;
    if (T == 0) return CZ_OK;
    cudaSetDevice(g.dev);
    uint8_t* base = noalloc_scratch(g.dev);
    if (!base) return CZ_ELAUNCH;
    uint32_t* sync = reinterpret_cast<uint32_t*>(base);
    unsigned long long* logits = reinterpret_cast<unsigned long long*>(base + kNoAllocSyncBytes);
    unsigned long long* hrows = reinterpret_cast<unsigned long long*>(base + kNoAllocSyncBytes + kNoAllocLogitBytes);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int bf16 = x_dtype == COLIZIG_X_BF16;
    const size_t xelt = bf16 ? 2 : 4;
    int tmax = cz::decode_max_tokens((int)L.d.hidden, (int)L.d.experts, (int)L.d.topk, (int)L.d.inter,
                                     (int)L.d.shared_inter, bf16, g.num_sms);
    if (tmax > kNoAllocMaxTokens) tmax = kNoAllocMaxTokens;
    if (tmax < 1) return CZ_ESHAPE;
    for (int t0 = 0; t0 < T; t0 += tmax) {
        const int n = T - t0 < tmax ? T - t0 : tmax;
        cz::DecodeParams p = make_params(L);
        p.logits = logits;
        p.hrows = hrows;
        p.sync = sync;
        p.x = reinterpret_cast<const uint8_t*>(x) + (size_t)t0 * L.d.hidden * xelt;
        p.x_bf16 = bf16;
        p.T = n;
        p.out = out + (size_t)t0 * L.d.hidden;
        p.topk_idx = topk_idx ? topk_idx + (size_t)t0 * L.d.topk : nullptr;
        p.topk_gates = topk_gates ? topk_gates + (size_t)t0 * L.d.topk : nullptr;
        take_debug_hold(p);
        const int rc = cz::decode_launch(p, g.num_sms, st);
        if (rc) return rc;
    }
    // Without a status the error word is kept: a wait that gave up stays recorded
    // until a later call passes a status (that call then reports it).
    if (status) {
        if (cudaMemcpyAsync(status, sync + 1, sizeof(uint32_t), cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            return CZ_ELAUNCH;
        if (cudaMemsetAsync(sync + 1, 0, sizeof(uint32_t), st) != cudaSuccess) return CZ_ELAUNCH;
    }
    return CZ_OK;
}
