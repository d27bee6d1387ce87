// hostpool.cu — page-locked host memory for the drop-in API's result arrays.
//
// The reference returns malloc'd arrays that the caller releases with the
// *_free functions (src/kv-compact-api.cpp:517-524,954-965,1231-1232). Fresh
// malloc'd memory is pageable and not yet faulted in, so copying ~100 MB of
// results per layer into it costs more than the compaction itself. Result
// arrays here come from a pool of page-locked blocks instead: the device
// writes into them directly at full link bandwidth, and *_free returns them
// to the pool, so the next call reuses memory that is already pinned and
// mapped. Blocks are kept in power-of-two size classes; the pool holds at
// most KVC_HOST_POOL_MB (default 4096) MiB, beyond which arrays fall back to
// malloc (and the staged copy path). kv_compact_cuda_pool_free() releases
// every cached block.
#include <stdlib.h>

#include <map>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "engine.h"

namespace {
struct host_pool {
    std::mutex mu;
    std::unordered_map<void *, size_t> owned;        // pinned block -> capacity (in use or cached)
    std::map<size_t, std::vector<void *>> free_by_cap;
    size_t total = 0;                                 // bytes of pinned blocks held
    size_t limit = 0;
};

host_pool & pool() {
    static host_pool * p = new host_pool();          // lives until exit (results may outlive statics)
    return *p;
}

size_t pool_limit() {
    const char * e = getenv("KVC_HOST_POOL_MB");
    long long mb = e ? atoll(e) : 4096;
    if (mb < 0) mb = 0;
    return (size_t)mb << 20;
}

size_t size_class(size_t bytes) {
    size_t c = 4096;
    while (c < bytes) c <<= 1;
    return c;
}
}  // namespace

void * kvc_hmalloc(size_t bytes) {
    if (bytes == 0) bytes = 1;
    host_pool & hp = pool();
    const size_t cap = size_class(bytes);
    {
        std::lock_guard<std::mutex> lk(hp.mu);
        if (hp.limit == 0) hp.limit = pool_limit() + 1;
        auto it = hp.free_by_cap.find(cap);
        if (it != hp.free_by_cap.end() && !it->second.empty()) {
            void * p = it->second.back();
            it->second.pop_back();
            return p;
        }
        if (hp.total + cap >= hp.limit) return malloc(bytes);
        hp.total += cap;                              // reserve before the (slow) allocation
    }
    void * p = nullptr;
    if (cudaHostAlloc(&p, cap, cudaHostAllocDefault) != cudaSuccess) {
        cudaGetLastError();
        std::lock_guard<std::mutex> lk(hp.mu);
        hp.total -= cap;
        return malloc(bytes);
    }
    std::lock_guard<std::mutex> lk(hp.mu);
    hp.owned[p] = cap;
    return p;
}

void kvc_hfree(void * p) {
    if (!p) return;
    host_pool & hp = pool();
    std::lock_guard<std::mutex> lk(hp.mu);
    auto it = hp.owned.find(p);
    if (it == hp.owned.end()) {
        free(p);
        return;
    }
    hp.free_by_cap[it->second].push_back(p);
}

bool kvc_is_pinned(const void * p) {
    host_pool & hp = pool();
    std::lock_guard<std::mutex> lk(hp.mu);
    return hp.owned.count(const_cast<void *>(p)) != 0;
}

// Release every cached (not in use) pinned block.
void kvc_hpool_release() {
    host_pool & hp = pool();
    std::lock_guard<std::mutex> lk(hp.mu);
    for (auto & kv : hp.free_by_cap) {
        for (void * p : kv.second) {
            hp.owned.erase(p);
            hp.total -= kv.first;
            cudaFreeHost(p);
        }
        kv.second.clear();
    }
}
