// Peer-memory groups over CUDA IPC (see fn_peer.h) and the row-split lm_head entry point.
//
// Setup, per rank (the host side exchanges the 64-byte handles, e.g. with torch.distributed):
//   fn_ipc_alloc(bytes) -> this rank's buffer + its handle; fn_ipc_open(peer handle) -> the peer's buffer mapped here;
//   fn_group_create(rank, n, bases) once every base is known. Teardown: fn_group_free, a host barrier, fn_ipc_free.
// Every rank must make the same sequence of exchange calls on a group (the counters count calls).
#include <cstring>
#include <mutex>
#include <vector>

#include "fn_peer.h"

namespace fn {

static std::vector<PeerGroup *> g_groups;
static std::mutex g_groups_mu;

PeerGroup *peer_group(int g) {
    std::lock_guard<std::mutex> l(g_groups_mu);
    return g >= 1 && g <= (int)g_groups.size() ? g_groups[g - 1] : nullptr;
}

KeyExchange key_exchange(const PeerGroup &pg) {
    KeyExchange x;
    x.n = pg.n;
    x.rank = pg.rank;
    for (int r = 0; r < pg.n; ++r) {
        x.keys[r] = (unsigned long long *)(pg.base[r] + PEER_KEYS);
        x.counters[r] = (uint32_t *)(pg.base[r] + PEER_KEY_COUNTERS);
    }
    x.calls = pg.local_calls;
    return x;
}

}  // namespace fn

using namespace fn;

// cudaMalloc `bytes` (zeroed) on the current device and export it: *ptr, handle[64]
FN_API int fn_ipc_alloc(size_t bytes, void **ptr, uint8_t *handle) {
    if (bytes < PEER_MIN_BYTES) bytes = PEER_MIN_BYTES;
    void *p = nullptr;
    FN_CK(cudaMalloc(&p, bytes));
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(std::string("fn_ipc_alloc: ") + cudaGetErrorString(e));
    }
    static_assert(sizeof(h) == 64, "IPC handle size");
    memcpy(handle, &h, 64);
    *ptr = p;
    return 0;
}

// map a peer's exported buffer into this process (peer access enabled on demand)
FN_API int fn_ipc_open(const uint8_t *handle, void **ptr) {
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, 64);
    FN_CK(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return 0;
}
FN_API int fn_ipc_close(void *ptr) {
    FN_CK(cudaIpcCloseMemHandle(ptr));
    return 0;
}
FN_API int fn_ipc_free(void *ptr) {
    FN_CK(cudaFree(ptr));
    return 0;
}

// group of n ranks over their buffers bases[n] (bases[rank] = this rank's fn_ipc_alloc buffer, the others opened with
// fn_ipc_open); every buffer at least `bytes`. Returns the group id (>= 1) or -1.
FN_API int fn_group_create(int rank, int n, void *const *bases, size_t bytes) {
    if (n < 1 || n > MAX_RANKS || rank < 0 || rank >= n || bytes < PEER_MIN_BYTES)
        return fail("fn_group_create: bad rank / size");
    PeerGroup *g = new PeerGroup();
    g->rank = rank;
    g->n = n;
    g->bytes = bytes;
    cudaGetDevice(&g->dev);
    for (int r = 0; r < n; ++r) {
        if (!bases[r]) {
            delete g;
            return fail("fn_group_create: missing buffer of rank " + std::to_string(r));
        }
        g->base[r] = (uint8_t *)bases[r];
    }
    if (cudaMalloc(&g->local_calls, 64) != cudaSuccess || cudaMemset(g->local_calls, 0, 64) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(g->local_calls);
        delete g;
        return fail("fn_group_create: device allocation failed");
    }
    std::lock_guard<std::mutex> l(g_groups_mu);
    g_groups.push_back(g);
    return (int)g_groups.size();
}

// forget a group (the buffers stay with their owners: fn_ipc_close / fn_ipc_free)
FN_API int fn_group_free(int gid) {
    PeerGroup *g = peer_group(gid);
    if (!g) return fail("fn_group_free: bad group");
    cudaFree(g->local_calls);
    delete g;
    std::lock_guard<std::mutex> l(g_groups_mu);
    g_groups[gid - 1] = nullptr;
    return 0;
}
