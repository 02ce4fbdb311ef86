// Device helpers of the expert-parallel exchange shared by ep_peer.cu and permute.cu: system-scope
// stamp loads/stores, the bounded wait for every peer's stamp, and the gather of the routes that land
// on this rank's experts from every peer's published id/weight tables.
#pragma once
#include "common.cuh"
#include "internal.h"

namespace dsv41 {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// thread 0 of the block waits until every peer's stamp in flags[0..world) reached `stamp`, at most
// limit_ns in all; returns false for the whole block on timeout (and records kStatusWaitTimeout)
__device__ __forceinline__ bool block_wait_stamps(const uint32_t* flags, int world, uint32_t stamp, int* status,
                                                  uint64_t limit_ns)
{
    __shared__ int ok;
    if (threadIdx.x == 0) {
        ok = 1;
        const uint64_t t0 = globaltimer_ns();
        for (int d = 0; d < world && ok; ++d) {
            uint32_t it = 0;
            while ((int)(ld_acquire_sys(flags + d) - stamp) < 0) {
                if ((++it & 63u) == 0 && globaltimer_ns() - t0 > limit_ns) {
                    atomicExch(status, kStatusWaitTimeout);
                    ok = 0;
                    break;
                }
            }
        }
    }
    __syncthreads();
    return ok != 0;
}

// routes i = t0, t0 + step, ... of the world * per gathered entries (entry d * per + r = route r of rank
// d): local expert id (e - lo for e in [lo, hi), else -1) and weight; with ok false every entry is -1.
// Each thread issues the peer loads of four entries (ids and weights) before it uses any of them.
__device__ __forceinline__ void ep_gather_routes(const EpGather& g, bool ok, long long t0, long long step)
{
    const long long n = (long long)g.per * g.world;
    for (long long i0 = t0; i0 < n; i0 += 4 * step) {
        int e[4];
        float wt[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const long long i = i0 + u * step;
            e[u] = -1;
            wt[u] = 0.0f;
            if (ok && i < n) {
                const int d = (int)(i / g.per);
                const long long r = i - (long long)d * g.per;
                const uint8_t* b = static_cast<const uint8_t*>(g.peers.base[d]);
                e[u] = __ldcg(reinterpret_cast<const int*>(b + g.ids_off) + r);
                wt[u] = __ldcg(reinterpret_cast<const float*>(b + g.w_off) + r);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const long long i = i0 + u * step;
            if (i >= n) break;
            const bool mine = e[u] >= g.lo && e[u] < g.hi;
            g.ids_out[i] = mine ? (int64_t)(e[u] - g.lo) : -1;
            g.w_out[i] = mine ? wt[u] : 0.0f;
        }
    }
}

}  // namespace dsv41
