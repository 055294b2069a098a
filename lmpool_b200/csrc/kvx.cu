// KV-cache data path for B200 (sm_100a): block moves within one GPU and
// pushes into a peer GPU's cache over NVLink, plus the store_kvcache scatter.
// Exposes the C ABI declared in include/kvx.h.
//
// Reference behaviour being replaced (LMPool, Python):
//   src/lmpool/engine/kv_transfer.py:229-276  pack/unpack of all layers
//   src/lmpool/engine/kv_transfer.py:395-475  swap_in, planned path
//   src/lmpool/layers/attention.py:7-108      store_kvcache
//
// Work decomposition of a move. A transfer of B blocks is 2 * L * B
// independent contiguous chunks (plane kv, layer l, block i), each
// chunk_bytes long (512 KiB at block_size 256, 32 KiB at block_size 16).
// Chunks are cut into tiles of tile_bytes; tile t of a segment decodes as
//   j = t % tiles_per_chunk, u = t / tiles_per_chunk,
//   i = u % B, kvl = u / B, l = kvl % L, kv = kvl / L.
// A persistent grid (a multiple of the SM count) walks the tiles with a
// CTA-stride loop. Two copy engines share that decomposition:
//   - register: every thread moves 4 x 16 B per step with non-coherent
//     streaming loads and evict-first stores;
//   - bulk: one thread per CTA drives a shared-memory ring with
//     cp.async.bulk loads (mbarrier completion) and cp.async.bulk stores
//     (bulk-group completion), the Blackwell copy unit doing the bytes.
// A push launch may carry several segments (destinations); each segment owns
// a contiguous CTA range so that all destinations progress together, and the
// last CTA of a segment publishes the completion token to that destination.

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_set>
#include <vector>

#include <cuda.h>
#include <cuda_runtime.h>

#include "kvx.h"
#include "kvx_device.cuh"

namespace kvx {

constexpr int kMaxSegments = 8;
constexpr int kRegThreads = 256;
constexpr int kRegUnroll = 4;
constexpr int kStoreThreads = 64;   // one token's K row and V row per CTA
constexpr int kMaxDevices = 64;
constexpr uint64_t kFailBit = 1ull << 63;
// Upper bound on mbarrier polls of a bulk-copy stage before the pipeline
// gives up (each poll may suspend for a hardware-chosen interval).
constexpr uint32_t kMaxPipePolls = 1u << 24;
// Segment completion counters count CTAs in the low 16 bits and failed CTAs
// in the high 16 bits (a grid never exceeds 148 SMs x 32 CTAs < 2^16).
constexpr unsigned kCtaOne = 1u;
constexpr unsigned kCtaFailed = 1u << 16;
constexpr unsigned kCtaMask = kCtaFailed - 1u;

struct SegParams {
    uint64_t dst_base;
    int64_t dst_kv_stride;
    int64_t dst_layer_stride;
    int64_t dst_block_stride;
    int64_t dst_num_blocks;
    const int64_t* src_ids;  // nullptr: identity
    const int64_t* dst_ids;  // nullptr: identity
    int64_t num_ids;
    int64_t num_tiles;
    const uint64_t* go;      // nullptr: always run; else run iff *go != 0 and signal *go
    // Grant check (pull): the segment copies only if *cond == cond_value when
    // it starts; otherwise it moves nothing and signals token | FAIL.
    const uint64_t* cond;
    uint64_t cond_value;
    unsigned int* counter;   // CTA completion counter (nullptr: no signal)
    uint64_t* flag;          // completion flag written by the segment's last CTA
    uint64_t token;          // token to signal when go is nullptr (pull)
    // Per-segment source (pull: each segment reads another peer's cache);
    // src_base == 0 means the launch-wide source in MoveParams.
    uint64_t src_base;
    int64_t src_kv_stride;
    int64_t src_layer_stride;
    int64_t src_block_stride;
    int64_t src_num_blocks;
    int32_t cta_begin;
    int32_t cta_count;
};

struct MoveParams {
    uint64_t src_base;
    int64_t src_kv_stride;
    int64_t src_layer_stride;
    int64_t src_block_stride;
    int64_t src_num_blocks;
    int64_t chunk_bytes;
    int64_t tile_bytes;
    int64_t tiles_per_chunk;
    int32_t num_layers;
    int32_t num_segs;
    int32_t* status;
    SegParams seg[kMaxSegments];
};

struct TileAddr {
    const char* src;
    char* dst;
    int64_t len;
    bool ok;
};

__device__ __forceinline__ int find_segment(const MoveParams& p) {
    int s = 0;
    while (s + 1 < p.num_segs && (int)blockIdx.x >= p.seg[s + 1].cta_begin) ++s;
    return s;
}

__device__ __forceinline__ TileAddr decode_tile(const MoveParams& p, const SegParams& g, int64_t t, bool report) {
    TileAddr a;
    const int64_t j = t % p.tiles_per_chunk;
    const int64_t u = t / p.tiles_per_chunk;
    const int64_t i = u % g.num_ids;
    const int64_t kvl = u / g.num_ids;
    const int64_t l = kvl % p.num_layers;
    const int64_t kv = kvl / p.num_layers;
    const int64_t sid = g.src_ids ? ld_id(g.src_ids + i) : i;
    const int64_t did = g.dst_ids ? ld_id(g.dst_ids + i) : i;
    const bool own_src = g.src_base != 0;
    const uint64_t src_base = own_src ? g.src_base : p.src_base;
    const int64_t src_kv = own_src ? g.src_kv_stride : p.src_kv_stride;
    const int64_t src_layer = own_src ? g.src_layer_stride : p.src_layer_stride;
    const int64_t src_block = own_src ? g.src_block_stride : p.src_block_stride;
    const int64_t src_blocks = own_src ? g.src_num_blocks : p.src_num_blocks;
    a.ok = true;
    if (sid < 0 || sid >= src_blocks) {
        if (report) atomicOr(p.status, KVX_DEV_BAD_SRC_ID);
        a.ok = false;
    }
    if (did < 0 || did >= g.dst_num_blocks) {
        if (report) atomicOr(p.status, KVX_DEV_BAD_DST_ID);
        a.ok = false;
    }
    const int64_t off = j * p.tile_bytes;
    a.len = min(p.tile_bytes, p.chunk_bytes - off);
    a.src = reinterpret_cast<const char*>(src_base + kv * src_kv + l * src_layer + sid * src_block + off);
    a.dst = reinterpret_cast<char*>(g.dst_base + kv * g.dst_kv_stride + l * g.dst_layer_stride +
                                    did * g.dst_block_stride + off);
    return a;
}

// CTA-cooperative copy of `bytes` (multiple of VEC, both pointers VEC-aligned).
template <int VEC>
__device__ __forceinline__ void copy_span(char* __restrict__ dst, const char* __restrict__ src, int64_t bytes) {
    using V = typename VecT<VEC>::T;
    const V* s = reinterpret_cast<const V*>(src);
    V* d = reinterpret_cast<V*>(dst);
    const int64_t n = bytes / VEC;
    const int64_t stride = blockDim.x;
    int64_t i = threadIdx.x;
    for (; i + (kRegUnroll - 1) * stride < n; i += kRegUnroll * stride) {
        V r[kRegUnroll];
#pragma unroll
        for (int k = 0; k < kRegUnroll; ++k) r[k] = ld_stream(s + i + k * stride);
#pragma unroll
        for (int k = 0; k < kRegUnroll; ++k) st_stream(d + i + k * stride, r[k]);
    }
    for (; i < n; i += stride) st_stream(d + i, ld_stream(s + i));
}

// Completion of one segment, called by one thread per CTA after the CTA's
// stores are fenced: every CTA counts itself in, failed or not; the last one
// release-stores the token into the flag (token | FAIL when any CTA of the
// segment failed or skipped its copy) and re-arms the counter, so a failure
// never leaves the counter part-way for the next transfer.
__device__ __forceinline__ void count_segment_cta(const SegParams& g, uint64_t token, bool failed) {
    const unsigned mine = kCtaOne + (failed ? kCtaFailed : 0u);
    const unsigned prev = atomicAdd(g.counter, mine);
    if ((prev & kCtaMask) == static_cast<unsigned>(g.cta_count) - 1u) {
        const bool any_failed = ((prev + mine) >> 16) != 0u;
        __threadfence_system();
        st_release_sys(g.flag, any_failed ? (token | kFailBit) : token);
        atomicExch(g.counter, 0u);
    }
}

// Whether the segment may copy: its grant word (pull) must carry exactly the
// token this transfer was granted under.
__device__ __forceinline__ bool segment_granted(const SegParams& g) {
    return g.cond == nullptr || ld_acquire_sys(g.cond) == g.cond_value;
}

template <int VEC>
__global__ void __launch_bounds__(kRegThreads) move_reg_kernel(const __grid_constant__ MoveParams p) {
    const int s = find_segment(p);
    const SegParams& g = p.seg[s];
    uint64_t token = g.token ? g.token : 1;
    if (g.go != nullptr) {
        token = ld_relaxed_gpu(g.go);
        if (token == 0) return;  // the arm wait failed: this segment does not run
    }
    __shared__ int granted;
    if (threadIdx.x == 0) granted = segment_granted(g) ? 1 : 0;
    __syncthreads();
    const int64_t local = static_cast<int64_t>(blockIdx.x) - g.cta_begin;
    if (granted) {
        for (int64_t t = local; t < g.num_tiles; t += g.cta_count) {
            const TileAddr a = decode_tile(p, g, t, threadIdx.x == 0);
            if (!a.ok) continue;
            copy_span<VEC>(a.dst, a.src, a.len);
        }
    }
    if (g.counter == nullptr) return;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) count_segment_cta(g, token, !granted);
}

// Bulk-copy engine: one warp per CTA, lane 0 issues everything. STAGES ring
// slots of tile_bytes each; loads run STAGES/2 tiles ahead of stores.
template <int STAGES>
__global__ void __launch_bounds__(32) move_bulk_kernel(const __grid_constant__ MoveParams p) {
    extern __shared__ __align__(1024) unsigned char smem[];
    if (threadIdx.x != 0) return;
    constexpr int kAhead = STAGES / 2;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    unsigned char* ring = smem + 1024;

    const int s = find_segment(p);
    const SegParams& g = p.seg[s];
    uint64_t token = g.token ? g.token : 1;
    if (g.go != nullptr) {
        token = ld_relaxed_gpu(g.go);
        if (token == 0) return;
    }
    const bool granted = segment_granted(g);
    for (int k = 0; k < STAGES; ++k) mbar_init(&bars[k], 1);
    mbar_init_fence();

    const int64_t local = static_cast<int64_t>(blockIdx.x) - g.cta_begin;
    const int64_t ntiles =
        (granted && local < g.num_tiles) ? (g.num_tiles - 1 - local) / g.cta_count + 1 : 0;
    char* dst_of[STAGES];
    uint32_t len_of[STAGES];
    bool ok_of[STAGES];

    auto issue_load = [&](int64_t k) {
        const int st = static_cast<int>(k % STAGES);
        const TileAddr a = decode_tile(p, g, local + k * g.cta_count, true);
        dst_of[st] = a.dst;
        len_of[st] = static_cast<uint32_t>(a.len);
        ok_of[st] = a.ok;
        if (a.ok) {
            mbar_arrive_expect_tx(&bars[st], static_cast<uint32_t>(a.len));
            bulk_load(ring + static_cast<int64_t>(st) * p.tile_bytes, a.src, static_cast<uint32_t>(a.len), &bars[st]);
        } else {
            mbar_arrive(&bars[st]);
        }
    };

    bool failed = false;
    const int64_t prologue = ntiles < kAhead ? ntiles : kAhead;
    for (int64_t k = 0; k < prologue; ++k) issue_load(k);
    for (int64_t k = 0; k < ntiles; ++k) {
        const int64_t kn = k + kAhead;
        if (kn < ntiles) {
            // Stage kn % STAGES last held tile kn - STAGES, whose store was
            // committed STAGES - kAhead groups ago: wait for its smem read.
            if (kn >= STAGES) bulk_wait_read<STAGES - kAhead - 1>();
            issue_load(kn);
        }
        const int st = static_cast<int>(k % STAGES);
        const uint32_t parity = static_cast<uint32_t>((k / STAGES) & 1);
        bool ready = false;
        for (uint32_t poll = 0; poll < kMaxPipePolls; ++poll) {
            if (mbar_try_wait(&bars[st], parity)) {
                ready = true;
                break;
            }
        }
        if (!ready) {
            atomicOr(p.status, KVX_DEV_PIPE_TIMEOUT);
            failed = true;
            // Loads of tiles k .. k + kAhead may still be in flight into this
            // CTA's shared memory: give each a second bounded wait before the
            // CTA leaves, so none lands after it exits.
            const int64_t last = (k + kAhead + 1 < ntiles ? k + kAhead + 1 : ntiles);
            for (int64_t kk = k; kk < last; ++kk) {
                const int sk = static_cast<int>(kk % STAGES);
                const uint32_t pk = static_cast<uint32_t>((kk / STAGES) & 1);
                for (uint32_t poll = 0; poll < kMaxPipePolls && !mbar_try_wait(&bars[sk], pk); ++poll) {
                }
            }
            break;
        }
        if (ok_of[st]) bulk_store(dst_of[st], ring + static_cast<int64_t>(st) * p.tile_bytes, len_of[st]);
        bulk_commit();
    }
    bulk_wait_all();
    if (g.counter == nullptr) return;
    fence_proxy_async();
    __threadfence_system();
    count_segment_cta(g, token, failed || !granted);
}

// ---------------------------------------------------------------------------
// Pair protocol kernels (one warp, lane 0 or the whole block as noted)
// ---------------------------------------------------------------------------

struct MailboxLayout {
    uint64_t arm, done, count, consumed, go, pulled, pull_consumed, granted, counter, pull_counter, ids, total;
};

// Per peer p: arm[p], count[p], ids[p][] (written by destination p, push),
// done[p] (written by source p, push), consumed[p], go[p] (local, push),
// pulled[p] (written by destination p after it pulled from this rank),
// pull_consumed[p] (local), granted[p] (local: the last token this rank
// granted to p), counter[p] / pull_counter[p] (CTA completion counters of
// this rank's push to p / pull from p).
__host__ __device__ inline MailboxLayout mailbox_layout(int64_t peers, int64_t max_blocks) {
    MailboxLayout m;
    m.arm = 0;
    m.done = m.arm + 8 * peers;
    m.count = m.done + 8 * peers;
    m.consumed = m.count + 8 * peers;
    m.go = m.consumed + 8 * peers;
    m.pulled = m.go + 8 * peers;
    m.pull_consumed = m.pulled + 8 * peers;
    m.granted = m.pull_consumed + 8 * peers;
    m.counter = m.granted + 8 * peers;
    m.pull_counter = m.counter + 4 * peers;
    m.ids = (m.pull_counter + 4 * peers + 255) / 256 * 256;
    m.total = m.ids + 8 * peers * max_blocks;
    return m;
}

// A pull request posts its block count with this tag, so that a source
// expecting a push (which needs target ids in its mailbox) and a source
// expecting a pull never accept each other's arm: the counts differ.
constexpr uint64_t kPullTag = 1ull << 62;

// Destination -> source mailbox: `n` target ids (push; none for a pull
// request), the count word, then the arm token.
__global__ void __launch_bounds__(1024) publish_kernel(const int64_t* ids, int64_t n, int64_t* remote_ids,
                                                         uint64_t count_word, uint64_t* remote_count,
                                                         uint64_t* remote_arm, uint64_t token) {
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) remote_ids[i] = ids[i];
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        st_relaxed_sys(remote_count, count_word);
        __threadfence_system();
        st_release_sys(remote_arm, token);
    }
}

// Source: wait for an arm newer than the last one consumed from this
// destination and check the posted count word.
//   push (go != nullptr): record the token the push will signal in *go
//     (0 = do not run); a count mismatch answers token | FAIL in remote_done.
//   grant (go == nullptr): record the token in *granted and answer it in
//     remote_done. The store
//     is ordered after every earlier kernel of this stream (they completed
//     before this one started, and the fence makes their writes visible to
//     the system), so the destination reads the blocks only after the
//     source's own writes to them.
__global__ void wait_armed_kernel(const uint64_t* arm, const uint64_t* count, uint64_t* consumed, uint64_t* go,
                                  uint64_t* granted, uint64_t* remote_done, uint64_t expected_count,
                                  uint64_t timeout_ns, int32_t* status) {
    if (threadIdx.x != 0) return;
    const uint64_t last = ld_relaxed_gpu(consumed);
    const uint64_t t0 = global_timer_ns();
    // Iteration cap as a second bound in case the timer does not advance.
    const uint64_t max_polls = timeout_ns / 64 + 1000000ull;
    for (uint64_t poll = 0; poll < max_polls; ++poll) {
        const uint64_t v = ld_acquire_sys(arm);
        if (v > last && (v & kFailBit) == 0) {
            const uint64_t n = ld_acquire_sys(count);
            *consumed = v;
            if (n != expected_count) {
                atomicOr(status, KVX_DEV_COUNT_MISMATCH);
                if (go != nullptr) *go = 0;
                __threadfence_system();
                st_release_sys(remote_done, v | kFailBit);
            } else if (go != nullptr) {
                *go = v;
            } else {
                if (granted != nullptr) *granted = v;
                __threadfence_system();
                st_release_sys(remote_done, v);
            }
            __threadfence();
            return;
        }
        if (global_timer_ns() - t0 > timeout_ns) break;
        __nanosleep(128);
    }
    if (go != nullptr) *go = 0;
    __threadfence();
    atomicOr(status, KVX_DEV_TIMEOUT);
}

// Destination: wait until the source's completion flag carries `token`.
__global__ void wait_done_kernel(const uint64_t* done, uint64_t token, uint64_t timeout_ns, int32_t* status) {
    if (threadIdx.x != 0) return;
    const uint64_t t0 = global_timer_ns();
    const uint64_t max_polls = timeout_ns / 64 + 1000000ull;
    for (uint64_t poll = 0; poll < max_polls; ++poll) {
        const uint64_t v = ld_acquire_sys(done);
        if ((v & ~kFailBit) == token) {
            if (v & kFailBit) atomicOr(status, KVX_DEV_PEER_FAILED);
            return;
        }
        if (global_timer_ns() - t0 > timeout_ns) break;
        __nanosleep(128);
    }
    atomicOr(status, KVX_DEV_TIMEOUT);
}

// Source (pull mode): wait until the destination reports a pull newer than
// the last one consumed from it and at least as new as the last token this
// rank granted it (so a report left over from an earlier transfer whose
// source did not wait for it never satisfies a newer one); FAIL bit -> the
// destination's pull failed.
__global__ void wait_pulled_kernel(const uint64_t* pulled, uint64_t* consumed, const uint64_t* granted,
                                   uint64_t timeout_ns, int32_t* status) {
    if (threadIdx.x != 0) return;
    const uint64_t last = ld_relaxed_gpu(consumed) & ~kFailBit;
    const uint64_t want = ld_relaxed_gpu(granted);
    const uint64_t t0 = global_timer_ns();
    const uint64_t max_polls = timeout_ns / 64 + 1000000ull;
    for (uint64_t poll = 0; poll < max_polls; ++poll) {
        const uint64_t v = ld_acquire_sys(pulled);
        const uint64_t token = v & ~kFailBit;
        if (token > last && token >= want) {
            *consumed = v;
            __threadfence();
            if (v & kFailBit) atomicOr(status, KVX_DEV_PEER_FAILED);
            return;
        }
        if (global_timer_ns() - t0 > timeout_ns) break;
        __nanosleep(128);
    }
    atomicOr(status, KVX_DEV_TIMEOUT);
}

__global__ void wait_flag_kernel(const uint64_t* flag, uint64_t expected, uint64_t timeout_ns, int32_t* status) {
    if (threadIdx.x != 0) return;
    const uint64_t t0 = global_timer_ns();
    const uint64_t max_polls = timeout_ns / 64 + 1000000ull;
    for (uint64_t poll = 0; poll < max_polls; ++poll) {
        if (ld_acquire_sys(flag) >= expected) return;
        if (global_timer_ns() - t0 > timeout_ns) break;
        __nanosleep(128);
    }
    atomicOr(status, KVX_DEV_TIMEOUT);
}

// ---------------------------------------------------------------------------
// store_kvcache: one warp per (token, plane), grid.y = layer
// ---------------------------------------------------------------------------

struct StoreParams {
    const char* key;
    const char* value;
    int64_t key_layer_stride;
    int64_t value_layer_stride;
    int64_t key_token_stride;
    int64_t value_token_stride;
    char* k_cache;
    char* v_cache;
    int64_t kc_layer_stride;
    int64_t vc_layer_stride;
    int64_t block_stride;
    int64_t slot_stride;
    const int64_t* slots;
    int64_t num_tokens;
    int64_t num_slots;
    int64_t row_bytes;
    int32_t block_size;
    int32_t* status;
};

// One warp per (token, plane), both planes of a token in one CTA, grid.y =
// layer. The token's row (up to 4 x 32 x VEC bytes; 2 KiB at H=8, D=128,
// VEC=16) is loaded before the slot id is tested, so the slot load and the
// row loads are in flight together; rows longer than that take a second loop.
// Launched with programmatic stream serialization: the slot id (an input of
// the whole step, written before the forward starts) is read before
// griddepcontrol.wait, K/V and the cache only after it, so everything the
// previous kernel wrote is visible; launch_dependents lets the next kernel
// (the next layer's store, when it uses the same launch) start its own
// prologue early. Without the launch attribute both instructions are no-ops.
template <int VEC>
__global__ void __launch_bounds__(kStoreThreads) store_kvcache_kernel(const __grid_constant__ StoreParams p) {
    using V = typename VecT<VEC>::T;
    constexpr int kUnroll = 4;
    griddep_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int64_t w = static_cast<int64_t>(blockIdx.x) * (kStoreThreads / 32) + (threadIdx.x >> 5);
    const int64_t t = w >> 1;
    const int kv = static_cast<int>(w & 1);
    if (t >= p.num_tokens) return;
    const int64_t layer = blockIdx.y;
    const int64_t slot = ld_cg(p.slots + t);
    griddep_wait();
    const char* src = kv ? p.value + layer * p.value_layer_stride + t * p.value_token_stride
                         : p.key + layer * p.key_layer_stride + t * p.key_token_stride;
    const V* s = reinterpret_cast<const V*>(src);
    const int64_t n = p.row_bytes / VEC;
    V r[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; ++k)
        if (lane + 32 * k < n) r[k] = ld_cg(s + lane + 32 * k);
    if (slot == -1) return;  // padding token (attention.py:29-30)
    if (slot < -1 || slot >= p.num_slots) {
        if (lane == 0 && kv == 0) atomicOr(p.status, KVX_DEV_BAD_SLOT);
        return;
    }
    const int64_t blk = slot / p.block_size;
    const int64_t off = slot - blk * p.block_size;
    char* dst = (kv ? p.v_cache + layer * p.vc_layer_stride : p.k_cache + layer * p.kc_layer_stride) +
                blk * p.block_stride + off * p.slot_stride;
    V* d = reinterpret_cast<V*>(dst);
#pragma unroll
    for (int k = 0; k < kUnroll; ++k)
        if (lane + 32 * k < n) d[lane + 32 * k] = r[k];
    for (int64_t i = lane + 32 * kUnroll; i < n; i += 32) d[i] = ld_cg(s + i);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(KVX_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define KVX_CUDA(call, what)                         \
    do {                                             \
        cudaError_t e_ = (call);                     \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    bool changed = false;
    cudaError_t err = cudaSuccess;
    explicit DeviceGuard(int dev) {
        err = cudaGetDevice(&prev);
        if (err == cudaSuccess && prev != dev) {
            err = cudaSetDevice(dev);
            changed = (err == cudaSuccess);
        }
    }
    ~DeviceGuard() {
        if (changed) cudaSetDevice(prev);
    }
};

#define KVX_DEVICE_GUARD(dev)                                            \
    DeviceGuard guard_(dev);                                             \
    if (guard_.err != cudaSuccess) return cuda_fail(guard_.err, "select device")

std::mutex g_mu;
kvx_tuning g_tuning = {0, 0, 0, 0, 0, 0};
int g_sm_count[kMaxDevices] = {0};
bool g_bulk_attr_set[kMaxDevices][4] = {};

int sm_count(int dev, int* out) {
    if (dev < 0 || dev >= kMaxDevices) return fail(KVX_EINVAL, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_sm_count[dev] == 0) {
        int n = 0;
        KVX_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev), "query SM count");
        g_sm_count[dev] = n;
    }
    *out = g_sm_count[dev];
    return KVX_OK;
}

int check_desc(const kvx_cache_desc* d, const char* name) {
    if (d == nullptr) return fail(KVX_EINVAL, "%s descriptor is NULL", name);
    if (d->base == 0) return fail(KVX_EINVAL, "%s.base is NULL", name);
    if (d->num_layers <= 0) return fail(KVX_EINVAL, "%s.num_layers must be > 0 (got %d)", name, d->num_layers);
    if (d->num_blocks <= 0) return fail(KVX_EINVAL, "%s.num_blocks must be > 0", name);
    if (d->chunk_bytes <= 0) return fail(KVX_EINVAL, "%s.chunk_bytes must be > 0", name);
    if (d->reserved != 0) return fail(KVX_EINVAL, "%s.reserved must be 0", name);
    return KVX_OK;
}

// Largest power-of-two vector width (<= 16) dividing every address term.
int pick_vec(const kvx_cache_desc* a, const std::vector<const kvx_cache_desc*>& others) {
    uint64_t bits = a->base | static_cast<uint64_t>(a->kv_stride) | static_cast<uint64_t>(a->layer_stride) |
                    static_cast<uint64_t>(a->block_stride) | static_cast<uint64_t>(a->chunk_bytes);
    for (auto* d : others)
        bits |= d->base | static_cast<uint64_t>(d->kv_stride) | static_cast<uint64_t>(d->layer_stride) |
                static_cast<uint64_t>(d->block_stride);
    for (int v = 16; v > 1; v >>= 1)
        if ((bits & static_cast<uint64_t>(v - 1)) == 0) return v;
    return 1;
}

struct LaunchPlan {
    int variant;  // 1 register, 2 bulk
    int vec;
    int grid;
    int stages;
    int64_t tile_bytes;
    size_t smem;
};

constexpr size_t kBulkMaxSmem = 227 * 1024;

// Opt in once per device to the largest ring any launch may use; each
// launch then passes its own (smaller or equal) dynamic shared memory size.
template <int S>
int set_bulk_attr(int dev, int idx) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_bulk_attr_set[dev][idx]) {
        KVX_CUDA(cudaFuncSetAttribute(move_bulk_kernel<S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(kBulkMaxSmem)),
                 "set bulk kernel shared memory");
        g_bulk_attr_set[dev][idx] = true;
    }
    return KVX_OK;
}

// Bulk ring depth when not tuned: measured on B200 at Qwen3-0.6B geometry,
// six 32 KiB stages reach 6.69 TB/s on 15 GB moves but four stages do
// better (3-4%) below a few GB, where the tail of the grid weighs more.
constexpr int64_t kDeepRingBytes = 4ll << 30;

int plan_launch(int dev, int vec, int64_t total_bytes, int64_t chunk_bytes, LaunchPlan* lp) {
    kvx_tuning t;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        t = g_tuning;
    }
    int sms = 0;
    int rc = sm_count(dev, &sms);
    if (rc) return rc;
    // Automatic choice: the bulk-copy engine wherever every address term is
    // 16-byte aligned (measured faster at every block count), else registers.
    int variant = t.variant;
    if (variant == 0) variant = (vec == 16) ? 2 : 1;
    if (variant == 2 && vec < 16) variant = 1;  // bulk copies need 16-byte granules
    lp->variant = variant;
    lp->vec = vec;
    if (variant == 1) {
        int64_t tile = t.tile_bytes > 0 ? t.tile_bytes : 32 * 1024;
        tile = std::max<int64_t>(vec, tile / vec * vec);
        lp->tile_bytes = std::min<int64_t>(tile, chunk_bytes);
        // 64 registers x 256 threads: 4 CTAs fill an SM's register file.
        const int cps = t.ctas_per_sm > 0 ? t.ctas_per_sm : 4;
        lp->grid = sms * cps;
        lp->stages = 0;
        lp->smem = 0;
    } else {
        int stages = t.stages > 0 ? t.stages : (total_bytes >= kDeepRingBytes ? 6 : 4);
        if (stages != 4 && stages != 6 && stages != 8 && stages != 12) stages = 6;
        int64_t tile = t.tile_bytes > 0 ? t.tile_bytes : 32 * 1024;
        tile = std::max<int64_t>(16, tile / 16 * 16);
        tile = std::min<int64_t>(tile, chunk_bytes);
        while (1024 + static_cast<size_t>(stages) * tile > kBulkMaxSmem && tile > 16) tile = (tile / 2 + 15) / 16 * 16;
        lp->tile_bytes = tile;
        lp->stages = stages;
        lp->smem = 1024 + static_cast<size_t>(stages) * tile;
        const int per_sm = std::max<int>(1, static_cast<int>((228 * 1024) / (lp->smem + 1024)));
        const int cps = t.ctas_per_sm > 0 ? std::min(t.ctas_per_sm, per_sm) : per_sm;
        lp->grid = sms * cps;
    }
    return KVX_OK;
}

int launch_move(int dev, MoveParams& p, const LaunchPlan& lp, cudaStream_t stream) {
    const dim3 grid(lp.grid);
    if (lp.variant == 1) {
        switch (lp.vec) {
            case 16: move_reg_kernel<16><<<grid, kRegThreads, 0, stream>>>(p); break;
            case 8: move_reg_kernel<8><<<grid, kRegThreads, 0, stream>>>(p); break;
            case 4: move_reg_kernel<4><<<grid, kRegThreads, 0, stream>>>(p); break;
            case 2: move_reg_kernel<2><<<grid, kRegThreads, 0, stream>>>(p); break;
            default: move_reg_kernel<1><<<grid, kRegThreads, 0, stream>>>(p); break;
        }
    } else {
        int rc = KVX_OK;
        switch (lp.stages) {
            case 4:
                rc = set_bulk_attr<4>(dev, 0);
                if (!rc) move_bulk_kernel<4><<<grid, 32, lp.smem, stream>>>(p);
                break;
            case 8:
                rc = set_bulk_attr<8>(dev, 2);
                if (!rc) move_bulk_kernel<8><<<grid, 32, lp.smem, stream>>>(p);
                break;
            case 12:
                rc = set_bulk_attr<12>(dev, 3);
                if (!rc) move_bulk_kernel<12><<<grid, 32, lp.smem, stream>>>(p);
                break;
            default:
                rc = set_bulk_attr<6>(dev, 1);
                if (!rc) move_bulk_kernel<6><<<grid, 32, lp.smem, stream>>>(p);
                break;
        }
        if (rc) return rc;
    }
    KVX_CUDA(cudaGetLastError(), "launch move kernel");
    return KVX_OK;
}

// Split `grid` CTAs across segments in proportion to their tiles; every
// segment gets at least one CTA and never more CTAs than tiles (a segment with
// no tiles keeps one CTA so that it still signals).
void assign_ctas(MoveParams& p, int grid) {
    int64_t total = 0;
    for (int s = 0; s < p.num_segs; ++s) total += p.seg[s].num_tiles;
    int begin = 0;
    for (int s = 0; s < p.num_segs; ++s) {
        int64_t share = total > 0 ? (static_cast<int64_t>(grid) * p.seg[s].num_tiles + total - 1) / total : 1;
        share = std::max<int64_t>(1, std::min<int64_t>(share, std::max<int64_t>(1, p.seg[s].num_tiles)));
        p.seg[s].cta_begin = begin;
        p.seg[s].cta_count = static_cast<int32_t>(share);
        begin += static_cast<int>(share);
    }
}

int total_ctas(const MoveParams& p) {
    return p.seg[p.num_segs - 1].cta_begin + p.seg[p.num_segs - 1].cta_count;
}

typedef CUresult (*PFN_getAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);

int get_alloc_base(const void* ptr, uint64_t* base, uint64_t* size) {
    static PFN_getAddressRange fn = nullptr;
    if (fn == nullptr) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        KVX_CUDA(cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 12000, cudaEnableDefault, &q),
                 "resolve cuMemGetAddressRange");
        if (f == nullptr || q != cudaDriverEntryPointSuccess)
            return fail(KVX_ECUDA, "cuMemGetAddressRange not available from the driver");
        fn = reinterpret_cast<PFN_getAddressRange>(f);
    }
    CUdeviceptr b = 0;
    size_t s = 0;
    CUresult r = fn(&b, &s, reinterpret_cast<CUdeviceptr>(ptr));
    if (r != CUDA_SUCCESS) return fail(KVX_EPEER, "cuMemGetAddressRange failed (CUresult %d)", static_cast<int>(r));
    *base = static_cast<uint64_t>(b);
    *size = static_cast<uint64_t>(s);
    return KVX_OK;
}

int check_mailbox(const kvx_mailbox* m, const char* name) {
    if (m == nullptr || m->base == 0) return fail(KVX_EINVAL, "%s mailbox is NULL", name);
    if (m->max_peers <= 0 || m->max_blocks <= 0) return fail(KVX_EINVAL, "%s mailbox has no capacity", name);
    if (m->reserved != 0) return fail(KVX_EINVAL, "%s mailbox reserved field must be 0", name);
    return KVX_OK;
}

template <typename T>
T* mb_ptr(const kvx_mailbox* m, uint64_t section_off, int64_t index) {
    return reinterpret_cast<T*>(m->base + section_off + sizeof(T) * index);
}

}  // namespace kvx

using namespace kvx;

extern "C" {

int kvx_abi_version(void) { return KVX_ABI_VERSION; }

const char* kvx_last_error(void) { return g_last_error; }

const char* kvx_status_name(int status) {
    switch (status) {
        case KVX_OK: return "KVX_OK";
        case KVX_EINVAL: return "KVX_EINVAL";
        case KVX_ENOMEM: return "KVX_ENOMEM";
        case KVX_ETIMEDOUT: return "KVX_ETIMEDOUT";
        case KVX_EPEER: return "KVX_EPEER";
        case KVX_ECUDA: return "KVX_ECUDA";
        case KVX_EUNSUPPORTED: return "KVX_EUNSUPPORTED";
        default: return "KVX_UNKNOWN";
    }
}

int kvx_set_tuning(const kvx_tuning* t) {
    if (t == nullptr) return fail(KVX_EINVAL, "tuning is NULL");
    if (t->variant < 0 || t->variant > 2) return fail(KVX_EINVAL, "variant must be 0, 1 or 2");
    if (t->ctas_per_sm < 0 || t->ctas_per_sm > 32) return fail(KVX_EINVAL, "ctas_per_sm must be in [0, 32]");
    if (t->tile_bytes < 0 || (t->tile_bytes % 16) != 0) return fail(KVX_EINVAL, "tile_bytes must be a multiple of 16");
    if (t->stages != 0 && t->stages != 4 && t->stages != 6 && t->stages != 8 && t->stages != 12)
        return fail(KVX_EINVAL, "stages must be 0, 4, 6, 8 or 12");
    if (t->store_pdl < 0 || t->store_pdl > 2) return fail(KVX_EINVAL, "store_pdl must be 0, 1 or 2");
    if (t->reserved != 0) return fail(KVX_EINVAL, "reserved must be 0");
    std::lock_guard<std::mutex> lk(g_mu);
    g_tuning = *t;
    return KVX_OK;
}

int kvx_get_tuning(kvx_tuning* out) {
    if (out == nullptr) return fail(KVX_EINVAL, "out is NULL");
    std::lock_guard<std::mutex> lk(g_mu);
    *out = g_tuning;
    return KVX_OK;
}

int kvx_validate_block_ids(const int64_t* ids, int64_t n, int64_t num_blocks, int32_t require_distinct) {
    if (n < 0) return fail(KVX_EINVAL, "negative id count");
    if (n > 0 && ids == nullptr) return fail(KVX_EINVAL, "ids is NULL");
    if (num_blocks <= 0) return fail(KVX_EINVAL, "num_blocks must be > 0");
    std::vector<uint8_t> seen;
    if (require_distinct) seen.assign(static_cast<size_t>(num_blocks), 0);
    for (int64_t i = 0; i < n; ++i) {
        const int64_t b = ids[i];
        if (b < 0 || b >= num_blocks)
            return fail(KVX_EINVAL, "block id %lld at position %lld is outside [0, %lld)", static_cast<long long>(b),
                        static_cast<long long>(i), static_cast<long long>(num_blocks));
        if (require_distinct) {
            if (seen[static_cast<size_t>(b)])
                return fail(KVX_EINVAL, "destination block id %lld appears more than once", static_cast<long long>(b));
            seen[static_cast<size_t>(b)] = 1;
        }
    }
    return KVX_OK;
}

int kvx_ids_overlap(const int64_t* a, int64_t na, const int64_t* b, int64_t nb, int64_t num_blocks,
                    int32_t* overlap_out) {
    if (overlap_out == nullptr) return fail(KVX_EINVAL, "overlap_out is NULL");
    if (num_blocks <= 0 || na < 0 || nb < 0) return fail(KVX_EINVAL, "bad sizes");
    std::vector<uint8_t> seen(static_cast<size_t>(num_blocks), 0);
    for (int64_t i = 0; i < na; ++i) {
        if (a[i] < 0 || a[i] >= num_blocks) return fail(KVX_EINVAL, "id %lld out of range", (long long)a[i]);
        seen[static_cast<size_t>(a[i])] = 1;
    }
    *overlap_out = 0;
    for (int64_t i = 0; i < nb; ++i) {
        if (b[i] < 0 || b[i] >= num_blocks) return fail(KVX_EINVAL, "id %lld out of range", (long long)b[i]);
        if (seen[static_cast<size_t>(b[i])]) {
            *overlap_out = 1;
            break;
        }
    }
    return KVX_OK;
}

int kvx_check_desc(const kvx_cache_desc* desc) { return check_desc(desc, "cache"); }

int kvx_device_count(int32_t* out) {
    if (out == nullptr) return fail(KVX_EINVAL, "out is NULL");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *out = 0;
        return cuda_fail(e, "cudaGetDeviceCount");
    }
    *out = n;
    return KVX_OK;
}

int kvx_device_sm_count(int32_t device, int32_t* out) {
    if (out == nullptr) return fail(KVX_EINVAL, "out is NULL");
    int n = 0;
    int rc = sm_count(device, &n);
    if (rc) return rc;
    *out = n;
    return KVX_OK;
}

int kvx_can_access_peer(int32_t device, int32_t peer, int32_t* out) {
    if (out == nullptr) return fail(KVX_EINVAL, "out is NULL");
    int v = 0;
    KVX_CUDA(cudaDeviceCanAccessPeer(&v, device, peer), "cudaDeviceCanAccessPeer");
    *out = v;
    return KVX_OK;
}

int kvx_move_blocks(int32_t device, const kvx_cache_desc* src, const kvx_cache_desc* dst, const int64_t* src_ids_dev,
                    const int64_t* dst_ids_dev, int64_t num_ids, int32_t* status_dev, void* stream) {
    int rc = check_desc(src, "src");
    if (rc) return rc;
    rc = check_desc(dst, "dst");
    if (rc) return rc;
    if (src->num_layers != dst->num_layers)
        return fail(KVX_EINVAL, "layer count differs: src %d, dst %d", src->num_layers, dst->num_layers);
    if (src->chunk_bytes != dst->chunk_bytes)
        return fail(KVX_EINVAL, "chunk size differs: src %lld, dst %lld", (long long)src->chunk_bytes,
                    (long long)dst->chunk_bytes);
    if (num_ids < 0) return fail(KVX_EINVAL, "negative block count");
    if (status_dev == nullptr) return fail(KVX_EINVAL, "status_dev is NULL");
    if (num_ids == 0) return KVX_OK;  // empty plan: nothing to move (kv_transfer.py:241-242, :211-212)
    KVX_DEVICE_GUARD(device);

    const int vec = pick_vec(src, {dst});
    LaunchPlan lp;
    rc = plan_launch(device, vec, num_ids * 2 * static_cast<int64_t>(src->num_layers) * src->chunk_bytes,
                     src->chunk_bytes, &lp);
    if (rc) return rc;

    MoveParams p;
    std::memset(&p, 0, sizeof(p));
    p.src_base = src->base;
    p.src_kv_stride = src->kv_stride;
    p.src_layer_stride = src->layer_stride;
    p.src_block_stride = src->block_stride;
    p.src_num_blocks = src->num_blocks;
    p.chunk_bytes = src->chunk_bytes;
    p.tile_bytes = lp.tile_bytes;
    p.tiles_per_chunk = (src->chunk_bytes + lp.tile_bytes - 1) / lp.tile_bytes;
    p.num_layers = src->num_layers;
    p.num_segs = 1;
    p.status = status_dev;
    SegParams& g = p.seg[0];
    g.dst_base = dst->base;
    g.dst_kv_stride = dst->kv_stride;
    g.dst_layer_stride = dst->layer_stride;
    g.dst_block_stride = dst->block_stride;
    g.dst_num_blocks = dst->num_blocks;
    g.src_ids = src_ids_dev;
    g.dst_ids = dst_ids_dev;
    g.num_ids = num_ids;
    g.num_tiles = num_ids * 2 * static_cast<int64_t>(src->num_layers) * p.tiles_per_chunk;
    assign_ctas(p, lp.grid);
    LaunchPlan run = lp;
    run.grid = total_ctas(p);
    return launch_move(device, p, run, static_cast<cudaStream_t>(stream));
}

int kvx_mailbox_bytes(int32_t max_peers, int64_t max_blocks, uint64_t* bytes_out) {
    if (bytes_out == nullptr) return fail(KVX_EINVAL, "bytes_out is NULL");
    if (max_peers <= 0 || max_blocks <= 0) return fail(KVX_EINVAL, "mailbox needs max_peers > 0 and max_blocks > 0");
    *bytes_out = mailbox_layout(max_peers, max_blocks).total;
    return KVX_OK;
}

int kvx_mailbox_create(int32_t device, int32_t max_peers, int64_t max_blocks, kvx_mailbox* out) {
    if (out == nullptr) return fail(KVX_EINVAL, "out is NULL");
    if (max_peers <= 0 || max_blocks <= 0) return fail(KVX_EINVAL, "mailbox needs max_peers > 0 and max_blocks > 0");
    KVX_DEVICE_GUARD(device);
    const MailboxLayout m = mailbox_layout(max_peers, max_blocks);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, m.total);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(KVX_ENOMEM, "mailbox allocation of %llu bytes failed: %s", (unsigned long long)m.total,
                    cudaGetErrorString(e));
    }
    KVX_CUDA(cudaMemset(p, 0, m.total), "zero mailbox");
    KVX_CUDA(cudaDeviceSynchronize(), "zero mailbox");
    out->base = reinterpret_cast<uint64_t>(p);
    out->max_peers = max_peers;
    out->reserved = 0;
    out->max_blocks = max_blocks;
    return KVX_OK;
}

int kvx_mailbox_destroy(int32_t device, const kvx_mailbox* mailbox) {
    int rc = check_mailbox(mailbox, "local");
    if (rc) return rc;
    KVX_DEVICE_GUARD(device);
    KVX_CUDA(cudaFree(reinterpret_cast<void*>(mailbox->base)), "free mailbox");
    return KVX_OK;
}

int kvx_mailbox_read_done(int32_t device, const kvx_mailbox* mailbox, int32_t src_rank, uint64_t* token_out) {
    int rc = check_mailbox(mailbox, "local");
    if (rc) return rc;
    if (token_out == nullptr) return fail(KVX_EINVAL, "token_out is NULL");
    if (src_rank < 0 || src_rank >= mailbox->max_peers) return fail(KVX_EINVAL, "src_rank out of range");
    KVX_DEVICE_GUARD(device);
    const MailboxLayout m = mailbox_layout(mailbox->max_peers, mailbox->max_blocks);
    KVX_CUDA(cudaMemcpy(token_out, mb_ptr<uint64_t>(mailbox, m.done, src_rank), 8, cudaMemcpyDeviceToHost),
             "read mailbox");
    return KVX_OK;
}

int kvx_pair_publish(int32_t device, const kvx_mailbox* src_mb, int32_t my_rank, const int64_t* dst_ids_dev,
                     int64_t num_ids, uint64_t token, void* stream) {
    int rc = check_mailbox(src_mb, "source");
    if (rc) return rc;
    if (my_rank < 0 || my_rank >= src_mb->max_peers) return fail(KVX_EINVAL, "my_rank out of range");
    if (num_ids < 0 || num_ids > src_mb->max_blocks)
        return fail(KVX_EINVAL, "%lld target ids exceed the source mailbox capacity %lld", (long long)num_ids,
                    (long long)src_mb->max_blocks);
    if (num_ids > 0 && dst_ids_dev == nullptr) return fail(KVX_EINVAL, "dst_ids_dev is NULL");
    if (token == 0 || (token & kFailBit)) return fail(KVX_EINVAL, "token must be in [1, 2^63)");
    KVX_DEVICE_GUARD(device);
    const MailboxLayout m = mailbox_layout(src_mb->max_peers, src_mb->max_blocks);
    int64_t* ids = mb_ptr<int64_t>(src_mb, m.ids, static_cast<int64_t>(my_rank) * src_mb->max_blocks);
    publish_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
        dst_ids_dev, num_ids, ids, static_cast<uint64_t>(num_ids), mb_ptr<uint64_t>(src_mb, m.count, my_rank),
        mb_ptr<uint64_t>(src_mb, m.arm, my_rank), token);
    KVX_CUDA(cudaGetLastError(), "launch publish kernel");
    return KVX_OK;
}

int kvx_pair_wait_done(int32_t device, const kvx_mailbox* my_mb, int32_t src_rank, uint64_t token,
                       uint64_t timeout_ns, int32_t* status_dev, void* stream) {
    int rc = check_mailbox(my_mb, "local");
    if (rc) return rc;
    if (src_rank < 0 || src_rank >= my_mb->max_peers) return fail(KVX_EINVAL, "src_rank out of range");
    if (status_dev == nullptr) return fail(KVX_EINVAL, "status_dev is NULL");
    KVX_DEVICE_GUARD(device);
    const MailboxLayout m = mailbox_layout(my_mb->max_peers, my_mb->max_blocks);
    wait_done_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(mb_ptr<uint64_t>(my_mb, m.done, src_rank), token,
                                                                      timeout_ns, status_dev);
    KVX_CUDA(cudaGetLastError(), "launch wait-done kernel");
    return KVX_OK;
}

int kvx_pair_wait_armed(int32_t device, const kvx_mailbox* my_mb, const kvx_mailbox* dst_mb, int32_t my_rank,
                        int32_t dst_rank, int64_t num_ids, uint64_t timeout_ns, int32_t* status_dev, void* stream) {
    int rc = check_mailbox(my_mb, "local");
    if (rc) return rc;
    rc = check_mailbox(dst_mb, "destination");
    if (rc) return rc;
    if (dst_rank < 0 || dst_rank >= my_mb->max_peers) return fail(KVX_EINVAL, "dst_rank out of range");
    if (my_rank < 0 || my_rank >= dst_mb->max_peers) return fail(KVX_EINVAL, "my_rank out of range");
    if (status_dev == nullptr) return fail(KVX_EINVAL, "status_dev is NULL");
    KVX_DEVICE_GUARD(device);
    const MailboxLayout m = mailbox_layout(my_mb->max_peers, my_mb->max_blocks);
    const MailboxLayout md = mailbox_layout(dst_mb->max_peers, dst_mb->max_blocks);
    wait_armed_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        mb_ptr<uint64_t>(my_mb, m.arm, dst_rank), mb_ptr<uint64_t>(my_mb, m.count, dst_rank),
        mb_ptr<uint64_t>(my_mb, m.consumed, dst_rank), mb_ptr<uint64_t>(my_mb, m.go, dst_rank), nullptr,
        mb_ptr<uint64_t>(dst_mb, md.done, my_rank), static_cast<uint64_t>(num_ids), timeout_ns, status_dev);
    KVX_CUDA(cudaGetLastError(), "launch wait-armed kernel");
    return KVX_OK;
}

int kvx_pair_request(int32_t device, const kvx_mailbox* src_mb, int32_t my_rank, int64_t num_ids, uint64_t token,
                     void* stream) {
    int rc = check_mailbox(src_mb, "source");
    if (rc) return rc;
    if (my_rank < 0 || my_rank >= src_mb->max_peers) return fail(KVX_EINVAL, "my_rank out of range");
    if (num_ids < 0 || num_ids > src_mb->max_blocks)
        return fail(KVX_EINVAL, "%lld blocks exceed the source mailbox capacity %lld", (long long)num_ids,
                    (long long)src_mb->max_blocks);
    if (token == 0 || (token & kFailBit)) return fail(KVX_EINVAL, "token must be in [1, 2^63)");
    KVX_DEVICE_GUARD(device);
    const MailboxLayout m = mailbox_layout(src_mb->max_peers, src_mb->max_blocks);
    publish_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        nullptr, 0, nullptr, static_cast<uint64_t>(num_ids) | kPullTag, mb_ptr<uint64_t>(src_mb, m.count, my_rank),
        mb_ptr<uint64_t>(src_mb, m.arm, my_rank), token);
    KVX_CUDA(cudaGetLastError(), "launch request kernel");
    return KVX_OK;
}

int kvx_pair_grant(int32_t device, const kvx_mailbox* my_mb, const kvx_mailbox* dst_mb, int32_t my_rank,
                   int32_t dst_rank, int64_t num_ids, uint64_t timeout_ns, int32_t* status_dev, void* stream) {
    int rc = check_mailbox(my_mb, "local");
    if (rc) return rc;
    rc = check_mailbox(dst_mb, "destination");
    if (rc) return rc;
    if (dst_rank < 0 || dst_rank >= my_mb->max_peers) return fail(KVX_EINVAL, "dst_rank out of range");
    if (my_rank < 0 || my_rank >= dst_mb->max_peers) return fail(KVX_EINVAL, "my_rank out of range");
    if (num_ids < 0) return fail(KVX_EINVAL, "negative block count");
    if (status_dev == nullptr) return fail(KVX_EINVAL, "status_dev is NULL");
    KVX_DEVICE_GUARD(device);
    const MailboxLayout m = mailbox_layout(my_mb->max_peers, my_mb->max_blocks);
    const MailboxLayout md = mailbox_layout(dst_mb->max_peers, dst_mb->max_blocks);
    wait_armed_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        mb_ptr<uint64_t>(my_mb, m.arm, dst_rank), mb_ptr<uint64_t>(my_mb, m.count, dst_rank),
        mb_ptr<uint64_t>(my_mb, m.consumed, dst_rank), nullptr, mb_ptr<uint64_t>(my_mb, m.granted, dst_rank),
        mb_ptr<uint64_t>(dst_mb, md.done, my_rank), static_cast<uint64_t>(num_ids) | kPullTag, timeout_ns,
        status_dev);
    KVX_CUDA(cudaGetLastError(), "launch grant kernel");
    return KVX_OK;
}

int kvx_mailbox_reset_peer(int32_t device, const kvx_mailbox* mailbox, int32_t peer, void* stream) {
    int rc = check_mailbox(mailbox, "local");
    if (rc) return rc;
    if (peer < 0 || peer >= mailbox->max_peers) return fail(KVX_EINVAL, "peer out of range");
    KVX_DEVICE_GUARD(device);
    const MailboxLayout m = mailbox_layout(mailbox->max_peers, mailbox->max_blocks);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const uint64_t words[] = {m.arm, m.done, m.count, m.consumed, m.go, m.pulled, m.pull_consumed, m.granted};
    for (uint64_t off : words)
        KVX_CUDA(cudaMemsetAsync(mb_ptr<uint64_t>(mailbox, off, peer), 0, sizeof(uint64_t), st), "reset mailbox");
    KVX_CUDA(cudaMemsetAsync(mb_ptr<unsigned int>(mailbox, m.counter, peer), 0, sizeof(unsigned int), st),
             "reset mailbox");
    KVX_CUDA(cudaMemsetAsync(mb_ptr<unsigned int>(mailbox, m.pull_counter, peer), 0, sizeof(unsigned int), st),
             "reset mailbox");
    return KVX_OK;
}

int kvx_pair_push(int32_t device, const kvx_cache_desc* src, const kvx_mailbox* my_mb, int32_t my_rank,
                  const kvx_push_target* targets, int32_t num_targets, int32_t* status_dev, void* stream) {
    int rc = check_desc(src, "src");
    if (rc) return rc;
    rc = check_mailbox(my_mb, "local");
    if (rc) return rc;
    if (targets == nullptr || num_targets <= 0 || num_targets > kMaxSegments)
        return fail(KVX_EINVAL, "num_targets must be in [1, %d]", kMaxSegments);
    if (status_dev == nullptr) return fail(KVX_EINVAL, "status_dev is NULL");
    std::vector<const kvx_cache_desc*> others;
    std::unordered_set<int> ranks;
    for (int s = 0; s < num_targets; ++s) {
        const kvx_push_target& t = targets[s];
        rc = check_desc(&t.dst, "target dst");
        if (rc) return rc;
        rc = check_mailbox(&t.dst_mailbox, "target");
        if (rc) return rc;
        if (t.dst.num_layers != src->num_layers || t.dst.chunk_bytes != src->chunk_bytes)
            return fail(KVX_EINVAL, "target %d geometry differs from the source cache", s);
        if (t.num_ids < 0 || t.num_ids > my_mb->max_blocks)
            return fail(KVX_EINVAL, "target %d: %lld ids exceed mailbox capacity", s, (long long)t.num_ids);
        if (t.num_ids > 0 && t.src_ids_dev == nullptr) return fail(KVX_EINVAL, "target %d: src ids NULL", s);
        if (t.dst_rank < 0 || t.dst_rank >= my_mb->max_peers || t.dst_rank == my_rank)
            return fail(KVX_EINVAL, "target %d: bad dst_rank %d", s, t.dst_rank);
        if (my_rank < 0 || my_rank >= t.dst_mailbox.max_peers) return fail(KVX_EINVAL, "my_rank out of range");
        if (!ranks.insert(t.dst_rank).second) return fail(KVX_EINVAL, "target rank %d listed twice", t.dst_rank);
        others.push_back(&t.dst);
    }
    KVX_DEVICE_GUARD(device);
    const int vec = pick_vec(src, others);
    int64_t total_bytes = 0;
    for (int s = 0; s < num_targets; ++s)
        total_bytes += targets[s].num_ids * 2 * static_cast<int64_t>(src->num_layers) * src->chunk_bytes;
    LaunchPlan lp;
    rc = plan_launch(device, vec, total_bytes, src->chunk_bytes, &lp);
    if (rc) return rc;

    const MailboxLayout m = mailbox_layout(my_mb->max_peers, my_mb->max_blocks);
    MoveParams p;
    std::memset(&p, 0, sizeof(p));
    p.src_base = src->base;
    p.src_kv_stride = src->kv_stride;
    p.src_layer_stride = src->layer_stride;
    p.src_block_stride = src->block_stride;
    p.src_num_blocks = src->num_blocks;
    p.chunk_bytes = src->chunk_bytes;
    p.tile_bytes = lp.tile_bytes;
    p.tiles_per_chunk = (src->chunk_bytes + lp.tile_bytes - 1) / lp.tile_bytes;
    p.num_layers = src->num_layers;
    p.num_segs = num_targets;
    p.status = status_dev;
    for (int s = 0; s < num_targets; ++s) {
        const kvx_push_target& t = targets[s];
        const MailboxLayout md = mailbox_layout(t.dst_mailbox.max_peers, t.dst_mailbox.max_blocks);
        SegParams& g = p.seg[s];
        g.dst_base = t.dst.base;
        g.dst_kv_stride = t.dst.kv_stride;
        g.dst_layer_stride = t.dst.layer_stride;
        g.dst_block_stride = t.dst.block_stride;
        g.dst_num_blocks = t.dst.num_blocks;
        g.src_ids = t.src_ids_dev;
        g.dst_ids = mb_ptr<int64_t>(my_mb, m.ids, static_cast<int64_t>(t.dst_rank) * my_mb->max_blocks);
        g.num_ids = t.num_ids;
        // An empty transfer still signals; give it one id slot of no tiles.
        g.num_tiles = t.num_ids * 2 * static_cast<int64_t>(src->num_layers) * p.tiles_per_chunk;
        if (t.num_ids == 0) g.num_ids = 1;
        g.go = mb_ptr<uint64_t>(my_mb, m.go, t.dst_rank);
        g.counter = mb_ptr<unsigned int>(my_mb, m.counter, t.dst_rank);
        g.flag = mb_ptr<uint64_t>(&t.dst_mailbox, md.done, my_rank);
    }
    assign_ctas(p, lp.grid);
    LaunchPlan run = lp;
    run.grid = total_ctas(p);
    return launch_move(device, p, run, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free push
// ---------------------------------------------------------------------------
// The push kernel's only scratch memory is one CTA-completion counter per
// destination rank. kvx_pair_push keeps it in the mailbox region (made by
// kvx_mailbox_create with cudaMalloc); kvx_pair_push_noalloc keeps it here,
// in file-scope device storage: KVX_NOALLOC_MAX_PEERS * 4 = 256 bytes that
// every GPU loading this library holds until the process exits. In host
// code the array's name is only a host-side stand-in; its device address is
// resolved per device with cudaGetSymbolAddress and passed to the kernel.
namespace kvx {

static __device__ __align__(256) unsigned int g_noalloc_counters[KVX_NOALLOC_MAX_PEERS];
static unsigned int* g_noalloc_counters_dev[kMaxDevices] = {};

// Device address of g_noalloc_counters on `dev` (which must be current),
// resolved on the first call per device.
static int noalloc_counters(int dev, unsigned int** out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_noalloc_counters_dev[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_counters);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_counters)");
        }
        g_noalloc_counters_dev[dev] = static_cast<unsigned int*>(p);
    }
    *out = g_noalloc_counters_dev[dev];
    return KVX_OK;
}

}  // namespace kvx

extern "C" {

int kvx_pair_push_noalloc(int32_t device, const kvx_cache_desc* src, const kvx_mailbox* my_mb, int32_t my_rank,
                          const kvx_push_target* targets, int32_t num_targets, int32_t* status_dev, void* stream) {
    int rc = check_desc(src, "src");
    if (rc) return rc;
    rc = check_mailbox(my_mb, "local");
    if (rc) return rc;
    if (targets == nullptr || num_targets <= 0 || num_targets > kMaxSegments)
        return fail(KVX_EINVAL, "num_targets must be in [1, %d]", kMaxSegments);
    if (status_dev == nullptr) return fail(KVX_EINVAL, "status_dev is NULL");
    if (device < 0 || device >= kMaxDevices) return fail(KVX_EINVAL, "device %d out of range", device);
    std::vector<const kvx_cache_desc*> others;
    std::unordered_set<int> ranks;
    for (int s = 0; s < num_targets; ++s) {
        const kvx_push_target& t = targets[s];
        if (t.dst_rank < 0 || t.dst_rank >= KVX_NOALLOC_MAX_PEERS)
            return fail(KVX_EINVAL,
                        "target %d: destination rank %d is beyond the %d ranks the allocation-free push "
                        "supports (its scratch is a fixed array); use kvx_pair_push",
                        s, t.dst_rank, KVX_NOALLOC_MAX_PEERS);
        rc = check_desc(&t.dst, "target dst");
        if (rc) return rc;
        rc = check_mailbox(&t.dst_mailbox, "target");
        if (rc) return rc;
        if (t.dst.num_layers != src->num_layers || t.dst.chunk_bytes != src->chunk_bytes)
            return fail(KVX_EINVAL, "target %d geometry differs from the source cache", s);
        if (t.num_ids < 0 || t.num_ids > my_mb->max_blocks)
            return fail(KVX_EINVAL, "target %d: %lld ids exceed mailbox capacity", s, (long long)t.num_ids);
        if (t.num_ids > 0 && t.src_ids_dev == nullptr) return fail(KVX_EINVAL, "target %d: src ids NULL", s);
        if (t.dst_rank >= my_mb->max_peers || t.dst_rank == my_rank)
            return fail(KVX_EINVAL, "target %d: bad dst_rank %d", s, t.dst_rank);
        if (my_rank < 0 || my_rank >= t.dst_mailbox.max_peers) return fail(KVX_EINVAL, "my_rank out of range");
        if (!ranks.insert(t.dst_rank).second) return fail(KVX_EINVAL, "target rank %d listed twice", t.dst_rank);
        others.push_back(&t.dst);
    }
    KVX_DEVICE_GUARD(device);
    unsigned int* counters = nullptr;
    rc = noalloc_counters(device, &counters);
    if (rc) return rc;
    const int vec = pick_vec(src, others);
    int64_t total_bytes = 0;
    for (int s = 0; s < num_targets; ++s)
        total_bytes += targets[s].num_ids * 2 * static_cast<int64_t>(src->num_layers) * src->chunk_bytes;
    LaunchPlan lp;
    rc = plan_launch(device, vec, total_bytes, src->chunk_bytes, &lp);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // The array keeps whatever the last call left; this launch's counters
    // must start at zero (stream-ordered, no allocation).
    for (int s = 0; s < num_targets; ++s)
        KVX_CUDA(cudaMemsetAsync(counters + targets[s].dst_rank, 0, sizeof(unsigned int), st),
                 "clear push counters");

    const MailboxLayout m = mailbox_layout(my_mb->max_peers, my_mb->max_blocks);
    MoveParams p;
    std::memset(&p, 0, sizeof(p));
    p.src_base = src->base;
    p.src_kv_stride = src->kv_stride;
    p.src_layer_stride = src->layer_stride;
    p.src_block_stride = src->block_stride;
    p.src_num_blocks = src->num_blocks;
    p.chunk_bytes = src->chunk_bytes;
    p.tile_bytes = lp.tile_bytes;
    p.tiles_per_chunk = (src->chunk_bytes + lp.tile_bytes - 1) / lp.tile_bytes;
    p.num_layers = src->num_layers;
    p.num_segs = num_targets;
    p.status = status_dev;
    for (int s = 0; s < num_targets; ++s) {
        const kvx_push_target& t = targets[s];
        const MailboxLayout md = mailbox_layout(t.dst_mailbox.max_peers, t.dst_mailbox.max_blocks);
        SegParams& g = p.seg[s];
        g.dst_base = t.dst.base;
        g.dst_kv_stride = t.dst.kv_stride;
        g.dst_layer_stride = t.dst.layer_stride;
        g.dst_block_stride = t.dst.block_stride;
        g.dst_num_blocks = t.dst.num_blocks;
        g.src_ids = t.src_ids_dev;
        g.dst_ids = mb_ptr<int64_t>(my_mb, m.ids, static_cast<int64_t>(t.dst_rank) * my_mb->max_blocks);
        g.num_ids = t.num_ids;
        g.num_tiles = t.num_ids * 2 * static_cast<int64_t>(src->num_layers) * p.tiles_per_chunk;
        if (t.num_ids == 0) g.num_ids = 1;
        g.go = mb_ptr<uint64_t>(my_mb, m.go, t.dst_rank);
        g.counter = counters + t.dst_rank;
        g.flag = mb_ptr<uint64_t>(&t.dst_mailbox, md.done, my_rank);
    }
    assign_ctas(p, lp.grid);
    LaunchPlan run = lp;
    run.grid = total_ctas(p);
    return launch_move(device, p, run, st);
}

int kvx_pair_pull(int32_t device, const kvx_cache_desc* dst, const kvx_mailbox* my_mb, int32_t my_rank,
                  const kvx_pull_source* sources, int32_t num_sources, int32_t* status_dev, void* stream) {
    int rc = check_desc(dst, "dst");
    if (rc) return rc;
    rc = check_mailbox(my_mb, "local");
    if (rc) return rc;
    if (sources == nullptr || num_sources <= 0 || num_sources > kMaxSegments)
        return fail(KVX_EINVAL, "num_sources must be in [1, %d]", kMaxSegments);
    if (status_dev == nullptr) return fail(KVX_EINVAL, "status_dev is NULL");
    if (my_rank < 0 || my_rank >= my_mb->max_peers) return fail(KVX_EINVAL, "my_rank out of range");
    std::vector<const kvx_cache_desc*> others;
    std::unordered_set<int> ranks;
    int64_t total_bytes = 0;
    for (int s = 0; s < num_sources; ++s) {
        const kvx_pull_source& src = sources[s];
        rc = check_desc(&src.src, "source");
        if (rc) return rc;
        rc = check_mailbox(&src.src_mailbox, "source");
        if (rc) return rc;
        if (src.src.num_layers != dst->num_layers || src.src.chunk_bytes != dst->chunk_bytes)
            return fail(KVX_EINVAL, "source %d geometry differs from the local cache", s);
        if (src.num_ids < 0) return fail(KVX_EINVAL, "source %d: negative block count", s);
        if (src.num_ids > 0 && (src.src_ids_dev == nullptr || src.dst_ids_dev == nullptr))
            return fail(KVX_EINVAL, "source %d: ids NULL", s);
        if (src.token == 0 || (src.token & kFailBit)) return fail(KVX_EINVAL, "source %d: token out of range", s);
        if (src.src_rank < 0 || src.src_rank >= my_mb->max_peers || src.src_rank == my_rank)
            return fail(KVX_EINVAL, "source %d: bad src_rank %d", s, src.src_rank);
        if (my_rank >= src.src_mailbox.max_peers) return fail(KVX_EINVAL, "my_rank beyond the source mailbox");
        if (!ranks.insert(src.src_rank).second) return fail(KVX_EINVAL, "source rank %d listed twice", src.src_rank);
        others.push_back(&src.src);
        total_bytes += src.num_ids * 2 * static_cast<int64_t>(dst->num_layers) * dst->chunk_bytes;
    }
    KVX_DEVICE_GUARD(device);
    const int vec = pick_vec(dst, others);
    LaunchPlan lp;
    rc = plan_launch(device, vec, total_bytes, dst->chunk_bytes, &lp);
    if (rc) return rc;

    const MailboxLayout m = mailbox_layout(my_mb->max_peers, my_mb->max_blocks);
    MoveParams p;
    std::memset(&p, 0, sizeof(p));
    const kvx_cache_desc& s0 = sources[0].src;
    p.src_base = s0.base;
    p.src_kv_stride = s0.kv_stride;
    p.src_layer_stride = s0.layer_stride;
    p.src_block_stride = s0.block_stride;
    p.src_num_blocks = s0.num_blocks;
    p.chunk_bytes = dst->chunk_bytes;
    p.tile_bytes = lp.tile_bytes;
    p.tiles_per_chunk = (dst->chunk_bytes + lp.tile_bytes - 1) / lp.tile_bytes;
    p.num_layers = dst->num_layers;
    p.num_segs = num_sources;
    p.status = status_dev;
    for (int s = 0; s < num_sources; ++s) {
        const kvx_pull_source& src = sources[s];
        const MailboxLayout ms = mailbox_layout(src.src_mailbox.max_peers, src.src_mailbox.max_blocks);
        SegParams& g = p.seg[s];
        g.src_base = src.src.base;
        g.src_kv_stride = src.src.kv_stride;
        g.src_layer_stride = src.src.layer_stride;
        g.src_block_stride = src.src.block_stride;
        g.src_num_blocks = src.src.num_blocks;
        g.dst_base = dst->base;
        g.dst_kv_stride = dst->kv_stride;
        g.dst_layer_stride = dst->layer_stride;
        g.dst_block_stride = dst->block_stride;
        g.dst_num_blocks = dst->num_blocks;
        g.src_ids = src.src_ids_dev;
        g.dst_ids = src.dst_ids_dev;
        g.num_ids = src.num_ids;
        // An empty transfer still signals; give it one id slot of no tiles.
        g.num_tiles = src.num_ids * 2 * static_cast<int64_t>(dst->num_layers) * p.tiles_per_chunk;
        if (src.num_ids == 0) g.num_ids = 1;
        g.go = nullptr;
        g.token = src.token;
        // Copy only under the source's grant of exactly this token
        // (kvx_pair_grant answered it into done[src_rank]).
        g.cond = mb_ptr<uint64_t>(my_mb, m.done, src.src_rank);
        g.cond_value = src.token;
        g.counter = mb_ptr<unsigned int>(my_mb, m.pull_counter, src.src_rank);
        g.flag = mb_ptr<uint64_t>(&src.src_mailbox, ms.pulled, my_rank);
    }
    assign_ctas(p, lp.grid);
    LaunchPlan run = lp;
    run.grid = total_ctas(p);
    return launch_move(device, p, run, static_cast<cudaStream_t>(stream));
}

int kvx_pair_wait_pulled(int32_t device, const kvx_mailbox* my_mb, int32_t dst_rank, uint64_t timeout_ns,
                         int32_t* status_dev, void* stream) {
    int rc = check_mailbox(my_mb, "local");
    if (rc) return rc;
    if (dst_rank < 0 || dst_rank >= my_mb->max_peers) return fail(KVX_EINVAL, "dst_rank out of range");
    if (status_dev == nullptr) return fail(KVX_EINVAL, "status_dev is NULL");
    KVX_DEVICE_GUARD(device);
    const MailboxLayout m = mailbox_layout(my_mb->max_peers, my_mb->max_blocks);
    wait_pulled_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        mb_ptr<uint64_t>(my_mb, m.pulled, dst_rank), mb_ptr<uint64_t>(my_mb, m.pull_consumed, dst_rank),
        mb_ptr<uint64_t>(my_mb, m.granted, dst_rank), timeout_ns, status_dev);
    KVX_CUDA(cudaGetLastError(), "launch wait-pulled kernel");
    return KVX_OK;
}

int kvx_ipc_export(int32_t device, const void* dev_ptr, void* handle_out_64, uint64_t* offset_out) {
    if (dev_ptr == nullptr || handle_out_64 == nullptr || offset_out == nullptr)
        return fail(KVX_EINVAL, "NULL argument");
    KVX_DEVICE_GUARD(device);
    uint64_t base = 0, size = 0;
    int rc = get_alloc_base(dev_ptr, &base, &size);
    if (rc) return rc;
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(KVX_EPEER,
                    "cudaIpcGetMemHandle failed (%s); the KV cache must come from cudaMalloc "
                    "(PyTorch: expandable_segments off)",
                    cudaGetErrorString(e));
    }
    static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
    std::memcpy(handle_out_64, &h, 64);
    *offset_out = reinterpret_cast<uint64_t>(dev_ptr) - base;
    return KVX_OK;
}

int kvx_ipc_open(int32_t device, const void* handle_64, uint64_t offset, uint64_t* ptr_out) {
    if (handle_64 == nullptr || ptr_out == nullptr) return fail(KVX_EINVAL, "NULL argument");
    KVX_DEVICE_GUARD(device);
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle_64, 64);
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(KVX_EPEER, "cudaIpcOpenMemHandle failed: %s", cudaGetErrorString(e));
    }
    *ptr_out = reinterpret_cast<uint64_t>(p) + offset;
    return KVX_OK;
}

int kvx_ipc_close(int32_t device, uint64_t ptr, uint64_t offset) {
    if (ptr == 0) return fail(KVX_EINVAL, "NULL pointer");
    KVX_DEVICE_GUARD(device);
    cudaError_t e = cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr - offset));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(KVX_EPEER, "cudaIpcCloseMemHandle failed: %s", cudaGetErrorString(e));
    }
    return KVX_OK;
}

int kvx_enable_peer_access(int32_t device, int32_t peer) {
    KVX_DEVICE_GUARD(device);
    cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        return KVX_OK;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(KVX_EPEER, "enable peer access %d -> %d: %s", device, peer, cudaGetErrorString(e));
    }
    return KVX_OK;
}

static int store_common(int32_t device, int32_t num_layers, const void* key, const void* value,
                        int64_t key_layer_stride, int64_t value_layer_stride, int64_t key_token_stride,
                        int64_t value_token_stride, void* k_cache, void* v_cache, int64_t kc_layer_stride,
                        int64_t vc_layer_stride, int64_t block_stride, int64_t slot_stride, const int64_t* slots,
                        int64_t num_tokens, int64_t num_blocks, int32_t block_size, int64_t row_bytes,
                        int32_t* status, void* stream) {
    if (num_tokens < 0) return fail(KVX_EINVAL, "negative token count");
    if (num_layers <= 0 || num_layers > 65535) return fail(KVX_EINVAL, "num_layers must be in [1, 65535]");
    if (block_size <= 0) return fail(KVX_EINVAL, "block_size must be > 0");
    if (num_blocks <= 0) return fail(KVX_EINVAL, "num_blocks must be > 0");
    if (row_bytes <= 0) return fail(KVX_EINVAL, "row_bytes must be > 0");
    if (status == nullptr) return fail(KVX_EINVAL, "status_dev is NULL");
    if (num_tokens == 0) return KVX_OK;
    if (!key || !value || !k_cache || !v_cache || !slots) return fail(KVX_EINVAL, "NULL tensor pointer");
    KVX_DEVICE_GUARD(device);
    StoreParams p;
    p.key = static_cast<const char*>(key);
    p.value = static_cast<const char*>(value);
    p.key_layer_stride = key_layer_stride;
    p.value_layer_stride = value_layer_stride;
    p.key_token_stride = key_token_stride;
    p.value_token_stride = value_token_stride;
    p.k_cache = static_cast<char*>(k_cache);
    p.v_cache = static_cast<char*>(v_cache);
    p.kc_layer_stride = kc_layer_stride;
    p.vc_layer_stride = vc_layer_stride;
    p.block_stride = block_stride;
    p.slot_stride = slot_stride;
    p.slots = slots;
    p.num_tokens = num_tokens;
    p.num_slots = num_blocks * block_size;
    p.row_bytes = row_bytes;
    p.block_size = block_size;
    p.status = status;
    const uint64_t bits = reinterpret_cast<uint64_t>(key) | reinterpret_cast<uint64_t>(value) |
                          reinterpret_cast<uint64_t>(k_cache) | reinterpret_cast<uint64_t>(v_cache) |
                          static_cast<uint64_t>(key_layer_stride) | static_cast<uint64_t>(value_layer_stride) |
                          static_cast<uint64_t>(key_token_stride) | static_cast<uint64_t>(value_token_stride) |
                          static_cast<uint64_t>(kc_layer_stride) | static_cast<uint64_t>(vc_layer_stride) |
                          static_cast<uint64_t>(block_stride) | static_cast<uint64_t>(slot_stride) |
                          static_cast<uint64_t>(row_bytes);
    int vec = 1;
    for (int v = 16; v > 1; v >>= 1)
        if ((bits & static_cast<uint64_t>(v - 1)) == 0) {
            vec = v;
            break;
        }
    const int64_t warps = 2 * num_tokens;
    const int64_t wpc = kStoreThreads / 32;
    const int64_t blocks = (warps + wpc - 1) / wpc;
    if (blocks > 0x7fffffff) return fail(KVX_EINVAL, "too many tokens");
    const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(num_layers));
    int pdl;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        pdl = g_tuning.store_pdl != 2;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kStoreThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e;
    switch (vec) {
        case 16: e = cudaLaunchKernelEx(&cfg, store_kvcache_kernel<16>, p); break;
        case 8: e = cudaLaunchKernelEx(&cfg, store_kvcache_kernel<8>, p); break;
        case 4: e = cudaLaunchKernelEx(&cfg, store_kvcache_kernel<4>, p); break;
        case 2: e = cudaLaunchKernelEx(&cfg, store_kvcache_kernel<2>, p); break;
        default: e = cudaLaunchKernelEx(&cfg, store_kvcache_kernel<1>, p); break;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cuda_fail(e, "launch store_kvcache kernel");
    }
    return KVX_OK;
}

int kvx_store_kvcache(int32_t device, const void* key_dev, const void* value_dev, int64_t key_token_stride,
                      int64_t value_token_stride, void* k_cache_dev, void* v_cache_dev, int64_t cache_block_stride,
                      int64_t cache_slot_stride, const int64_t* slot_mapping_dev, int64_t num_tokens,
                      int64_t num_blocks, int32_t block_size, int64_t row_bytes, int32_t* status_dev, void* stream) {
    return store_common(device, 1, key_dev, value_dev, 0, 0, key_token_stride, value_token_stride, k_cache_dev,
                        v_cache_dev, 0, 0, cache_block_stride, cache_slot_stride, slot_mapping_dev, num_tokens,
                        num_blocks, block_size, row_bytes, status_dev, stream);
}

int kvx_store_kvcache_layers(int32_t device, int32_t num_layers, const void* key_dev, const void* value_dev,
                             int64_t key_layer_stride, int64_t value_layer_stride, int64_t key_token_stride,
                             int64_t value_token_stride, void* k_cache_dev, void* v_cache_dev,
                             int64_t k_cache_layer_stride, int64_t v_cache_layer_stride, int64_t cache_block_stride,
                             int64_t cache_slot_stride, const int64_t* slot_mapping_dev, int64_t num_tokens,
                             int64_t num_blocks, int32_t block_size, int64_t row_bytes, int32_t* status_dev,
                             void* stream) {
    return store_common(device, num_layers, key_dev, value_dev, key_layer_stride, value_layer_stride,
                        key_token_stride, value_token_stride, k_cache_dev, v_cache_dev, k_cache_layer_stride,
                        v_cache_layer_stride, cache_block_stride, cache_slot_stride, slot_mapping_dev, num_tokens,
                        num_blocks, block_size, row_bytes, status_dev, stream);
}

int kvx_wait_flag(int32_t device, const uint64_t* flag_dev, uint64_t expected, uint64_t timeout_ns,
                  int32_t* status_dev, void* stream) {
    if (flag_dev == nullptr || status_dev == nullptr) return fail(KVX_EINVAL, "NULL argument");
    KVX_DEVICE_GUARD(device);
    wait_flag_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flag_dev, expected, timeout_ns, status_dev);
    KVX_CUDA(cudaGetLastError(), "launch wait-flag kernel");
    return KVX_OK;
}

}  // extern "C"
