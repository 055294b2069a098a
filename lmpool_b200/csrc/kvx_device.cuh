// Device-side building blocks for the KV data path on sm_100a: vector
// load/store with cache hints, bulk-copy (TMA) and mbarrier wrappers,
// system-scope flag operations and the global timer. Everything here is
// inline PTX that this project wrote against the public PTX ISA; nothing is
// taken from a vendor binary.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "kvx.h"

namespace kvx {

// ---------------------------------------------------------------------------
// Vector types and loads/stores
// ---------------------------------------------------------------------------

template <int VEC>
struct VecT;
template <>
struct VecT<16> { using T = uint4; };
template <>
struct VecT<8> { using T = uint2; };
template <>
struct VecT<4> { using T = uint32_t; };
template <>
struct VecT<2> { using T = uint16_t; };
template <>
struct VecT<1> { using T = uint8_t; };

// Read-only streaming load: the source blocks are not written while a move
// runs (callers keep source and destination chunks disjoint), so the
// non-coherent path is valid; no_allocate keeps the once-read bytes out of L1.
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ld_stream(const uint2* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ld_stream(const uint32_t* p) { return __ldg(p); }
__device__ __forceinline__ uint16_t ld_stream(const uint16_t* p) { return __ldg(p); }
__device__ __forceinline__ uint8_t ld_stream(const uint8_t* p) { return __ldg(p); }

// Streaming store: evict-first in L2, the moved blocks are not re-read by
// this GPU soon. For peer addresses the hint is carried to the owner.
__device__ __forceinline__ void st_stream(uint4* p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ void st_stream(uint2* p, uint2 v) {
    asm volatile("st.global.cs.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}
__device__ __forceinline__ void st_stream(uint32_t* p, uint32_t v) { *p = v; }
__device__ __forceinline__ void st_stream(uint16_t* p, uint16_t v) { *p = v; }
__device__ __forceinline__ void st_stream(uint8_t* p, uint8_t v) { *p = v; }

// Load cached at L2 only (never from a possibly stale L1 line): rows written
// by the kernel just before this one, which may still have been running
// when this one started (programmatic dependent launch).
__device__ __forceinline__ uint4 ld_cg(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ld_cg(const uint2* p) {
    uint2 v;
    asm volatile("ld.global.cg.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ld_cg(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint16_t ld_cg(const uint16_t* p) {
    uint16_t v;
    asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint8_t ld_cg(const uint8_t* p) {
    uint16_t v;
    asm volatile("ld.global.cg.u8 %0, [%1];" : "=h"(v) : "l"(p));
    return static_cast<uint8_t>(v);
}
__device__ __forceinline__ int64_t ld_cg(const int64_t* p) {
    int64_t v;
    asm volatile("ld.global.cg.s64 %0, [%1];" : "=l"(v) : "l"(p));
    return v;
}

// Programmatic dependent launch (sm_90+): let the next kernel on the stream
// begin launching, and wait until every kernel before this one completed
// and its memory is visible. No-ops when the launch did not opt in.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Block ids may have been written by a peer GPU (target ids posted into this
// rank's mailbox) before this kernel started: read them at L2 (coherence
// point for this GPU's memory), never from a possibly stale L1 line.
__device__ __forceinline__ int64_t ld_id(const int64_t* p) {
    int64_t v;
    asm volatile("ld.global.cg.s64 %0, [%1];" : "=l"(v) : "l"(p));
    return v;
}

// ---------------------------------------------------------------------------
// Flags, fences and time
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t ld_relaxed_gpu(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------
// Bulk copy (TMA, non-tensor form) and mbarrier
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
// Make barrier initialisation visible to the async proxy (the bulk-copy unit
// completes transactions on these barriers).
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// global -> shared, completion counted in bytes on `bar`.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
// shared -> global (local HBM or a peer mapping), tracked by bulk groups.
__device__ __forceinline__ void bulk_store(void* gdst, const void* smem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_addr(smem_src)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async;" ::: "memory"); }

}  // namespace kvx
