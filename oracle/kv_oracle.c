/*
 * kv_oracle.c -- CPU restatement of LMPool's KV data path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA path and
 * the timed CPU baseline; it is never part of the product. Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
 *
 * Each function restates one piece of the reference (LMPool, Python/Triton),
 * byte for byte, on host memory:
 *   kvo_pack_all_layer_blocks    src/lmpool/engine/kv_transfer.py:229-248
 *   kvo_unpack_all_layer_blocks  src/lmpool/engine/kv_transfer.py:264-276, :199-215
 *   kvo_swap_planned             src/lmpool/engine/kv_transfer.py:395-475
 *                                (negotiate_blocks=False: pack on the source,
 *                                 one send/recv of the payload, unpack on
 *                                 the destination)
 *   kvo_store_kvcache            src/lmpool/layers/attention.py:7-64
 *
 * Layout convention (bytes): block b of layer l, plane kv starts at
 *   base + kv*kv_stride + l*layer_stride + b*block_stride
 * and is chunk_bytes long. The packed payload is [L, 2, B, chunk] contiguous,
 * as allocated at kv_transfer.py:236-240.
 *
 * Copies are split across `nthreads` POSIX threads by (layer, plane, block)
 * chunk; the result does not depend on the thread count because every chunk
 * has exactly one writer (destination ids are distinct, checked first).
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct kvo_layout {
    int64_t kv_stride;
    int64_t layer_stride;
    int64_t block_stride;
    int64_t num_blocks;
    int64_t chunk_bytes;
    int32_t num_layers;
    int32_t reserved;
} kvo_layout;

enum { KVO_OK = 0, KVO_EINVAL = 1, KVO_ENOMEM = 2 };

static int ids_in_range(const int64_t* ids, int64_t n, int64_t num_blocks) {
    for (int64_t i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= num_blocks) return 0;
    return 1;
}

static int ids_distinct(const int64_t* ids, int64_t n, int64_t num_blocks) {
    unsigned char* seen = (unsigned char*)calloc((size_t)num_blocks, 1);
    if (!seen) return 0;
    int ok = 1;
    for (int64_t i = 0; i < n && ok; ++i) {
        if (seen[ids[i]]) ok = 0;
        seen[ids[i]] = 1;
    }
    free(seen);
    return ok;
}

/* One copy job: chunks [begin, end) of a (layer, plane, block) enumeration. */
typedef struct job {
    const uint8_t* src_base;
    uint8_t* dst_base;
    const kvo_layout* src;  /* NULL: payload layout */
    const kvo_layout* dst;  /* NULL: payload layout */
    const int64_t* src_ids;
    const int64_t* dst_ids;
    int64_t n;
    int64_t chunk;
    int32_t layers;
    int64_t begin, end;
} job;

static int64_t payload_offset(int64_t l, int64_t kv, int64_t i, int64_t n, int64_t chunk) {
    return ((l * 2 + kv) * n + i) * chunk;
}

static void* run_job(void* arg) {
    job* j = (job*)arg;
    for (int64_t c = j->begin; c < j->end; ++c) {
        /* Enumeration order (layer, plane, block) follows the reference's
         * loops: for layer: K index op, then V index op. */
        const int64_t i = c % j->n;
        const int64_t kv = (c / j->n) % 2;
        const int64_t l = c / (2 * j->n);
        int64_t so, dof;
        if (j->src)
            so = kv * j->src->kv_stride + l * j->src->layer_stride + j->src_ids[i] * j->src->block_stride;
        else
            so = payload_offset(l, kv, i, j->n, j->chunk);
        if (j->dst)
            dof = kv * j->dst->kv_stride + l * j->dst->layer_stride + j->dst_ids[i] * j->dst->block_stride;
        else
            dof = payload_offset(l, kv, i, j->n, j->chunk);
        memcpy(j->dst_base + dof, j->src_base + so, (size_t)j->chunk);
    }
    return NULL;
}

static int run_parallel(job proto, int64_t total, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (total < nthreads) nthreads = total > 0 ? (int)total : 1;
    job jobs[256];
    pthread_t th[256];
    int started = 0;
    for (int t = 0; t < nthreads; ++t) {
        jobs[t] = proto;
        jobs[t].begin = total * t / nthreads;
        jobs[t].end = total * (t + 1) / nthreads;
    }
    if (nthreads == 1) {
        run_job(&jobs[0]);
        return KVO_OK;
    }
    for (int t = 0; t < nthreads; ++t) {
        if (pthread_create(&th[t], NULL, run_job, &jobs[t]) != 0) break;
        ++started;
    }
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
    /* Any job that could not get a thread runs here. */
    for (int t = started; t < nthreads; ++t) run_job(&jobs[t]);
    return KVO_OK;
}

/* _pack_all_layer_blocks: payload[l, kv, i] = cache[kv, l, ids[i]].
 * Source ids may repeat (index_select). */
int kvo_pack_all_layer_blocks(const uint8_t* cache, const kvo_layout* lay, const int64_t* ids, int64_t n,
                              uint8_t* payload, int32_t nthreads) {
    if (!cache || !lay || (n > 0 && (!ids || !payload)) || n < 0) return KVO_EINVAL;
    if (n == 0) return KVO_OK; /* kv_transfer.py:241-242 */
    if (!ids_in_range(ids, n, lay->num_blocks)) return KVO_EINVAL;
    job j = {cache, payload, lay, NULL, ids, NULL, n, lay->chunk_bytes, lay->num_layers, 0, 0};
    return run_parallel(j, (int64_t)lay->num_layers * 2 * n, nthreads);
}

/* _unpack_all_layer_blocks: cache[kv, l, ids[i]] = payload[l, kv, i].
 * Destination ids must be distinct (index_copy_ with repeated indices has
 * no defined result; LMPool's BlockManager never reserves a block twice). */
int kvo_unpack_all_layer_blocks(const uint8_t* payload, int64_t n, uint8_t* cache, const kvo_layout* lay,
                                const int64_t* ids, int32_t nthreads) {
    if (!cache || !lay || (n > 0 && (!ids || !payload)) || n < 0) return KVO_EINVAL;
    if (n == 0) return KVO_OK; /* kv_transfer.py:211-212 */
    if (!ids_in_range(ids, n, lay->num_blocks) || !ids_distinct(ids, n, lay->num_blocks)) return KVO_EINVAL;
    job j = {payload, cache, NULL, lay, NULL, ids, n, lay->chunk_bytes, lay->num_layers, 0, 0};
    return run_parallel(j, (int64_t)lay->num_layers * 2 * n, nthreads);
}

/* Planned swap_in: source packs, the payload crosses (here: one buffer that
 * stands for the NCCL send/recv), destination unpacks. src_cache and
 * dst_cache may be the same memory; the staging payload makes overlapping
 * id sets well defined, exactly as in the reference. `payload` must hold
 * L*2*n*chunk bytes (NULL: allocated here). */
int kvo_swap_planned(const uint8_t* src_cache, const kvo_layout* src_lay, const int64_t* src_ids,
                     uint8_t* dst_cache, const kvo_layout* dst_lay, const int64_t* dst_ids, int64_t n,
                     uint8_t* payload, int32_t nthreads) {
    if (!src_lay || !dst_lay) return KVO_EINVAL;
    if (src_lay->num_layers != dst_lay->num_layers || src_lay->chunk_bytes != dst_lay->chunk_bytes)
        return KVO_EINVAL;
    if (n == 0) return KVO_OK;
    uint8_t* own = NULL;
    if (!payload) {
        own = (uint8_t*)malloc((size_t)src_lay->num_layers * 2 * (size_t)n * (size_t)src_lay->chunk_bytes);
        if (!own) return KVO_ENOMEM;
        payload = own;
    }
    int rc = kvo_pack_all_layer_blocks(src_cache, src_lay, src_ids, n, payload, nthreads);
    if (rc == KVO_OK) rc = kvo_unpack_all_layer_blocks(payload, n, dst_cache, dst_lay, dst_ids, nthreads);
    free(own);
    return rc;
}

/* store_kvcache (attention.py:24-64): for each token t with
 * slot = slots[t] != -1, cache row (slot / block_size, slot % block_size)
 * receives key[t] (all heads, row_bytes bytes); the same for value.
 * Out-of-range slots (< -1 or >= num_blocks*block_size) make the Triton
 * kernel write out of bounds; here they are skipped and counted in
 * *bad_slots_out. */
int kvo_store_kvcache(const uint8_t* key, const uint8_t* value, int64_t key_token_stride, int64_t value_token_stride,
                      uint8_t* k_cache, uint8_t* v_cache, int64_t block_stride, int64_t slot_stride,
                      const int64_t* slots, int64_t num_tokens, int64_t num_blocks, int64_t block_size,
                      int64_t row_bytes, int64_t* bad_slots_out) {
    if (num_tokens < 0 || block_size <= 0 || num_blocks <= 0 || row_bytes <= 0) return KVO_EINVAL;
    int64_t bad = 0;
    for (int64_t t = 0; t < num_tokens; ++t) {
        const int64_t slot = slots[t];
        if (slot == -1) continue; /* attention.py:29-30 */
        if (slot < -1 || slot >= num_blocks * block_size) {
            ++bad;
            continue;
        }
        const int64_t blk = slot / block_size; /* attention.py:33-34 */
        const int64_t off = slot % block_size;
        const int64_t dst = blk * block_stride + off * slot_stride;
        memcpy(k_cache + dst, key + t * key_token_stride, (size_t)row_bytes);
        memcpy(v_cache + dst, value + t * value_token_stride, (size_t)row_bytes);
    }
    if (bad_slots_out) *bad_slots_out = bad;
    return KVO_OK;
}
