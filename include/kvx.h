/*
 * kvx.h -- C ABI of the B200 (sm_100a) KV-cache data path for LMPool.
 *
 * This library replaces the byte-moving parts of LMPool's cross-GPU KV
 * transfer and its store_kvcache scatter:
 *
 *   reference (LMPool, Python)                         this library
 *   -------------------------------------------------  ------------------------------
 *   kv_transfer.py:229-248 _pack_all_layer_blocks      kvx_move_blocks (dst = payload)
 *   kv_transfer.py:264-276 _unpack_all_layer_blocks    kvx_move_blocks (src = payload)
 *   kv_transfer.py:395-475 swap_in (planned path,      pull (default): kvx_pair_request +
 *     negotiate_blocks=False): index_select ->           kvx_pair_wait_done + kvx_pair_pull
 *     NCCL send/recv -> index_copy_                      (destination), kvx_pair_grant
 *                                                        [+ kvx_pair_wait_pulled] (source);
 *                                                        push: kvx_pair_publish +
 *                                                        kvx_pair_wait_done (destination),
 *                                                        kvx_pair_wait_armed + kvx_pair_push
 *                                                        (source)
 *   kv_transfer.py:40-119 prewarm_p2p_pairs            kvx_ipc_export / kvx_ipc_open /
 *     (pair NCCL communicators)                          kvx_mailbox_create
 *   layers/attention.py:7-108 store_kvcache            kvx_store_kvcache,
 *                                                        kvx_store_kvcache_layers
 *
 * Conventions
 *   - Every function returns an int status: KVX_OK (0) or one of the KVX_E*
 *     codes below. kvx_last_error() returns a message for the calling
 *     thread's last failure.
 *   - Pointers whose name ends in _dev are device addresses. All sizes,
 *     strides and offsets are in BYTES unless the name says otherwise.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream). Launching functions enqueue work and return without waiting;
 *     device-side failures are OR-ed as KVX_DEV_* bits into a caller-owned
 *     int32 status word (`status_dev`), which the caller reads after the
 *     stream completes.
 *   - No function here allocates device memory except kvx_mailbox_create.
 *
 * Memory layout served (LMPool model_runner.py:397-406): one tensor
 * [2, L, N, block_size, kv_heads, head_dim]; layer l's k_cache is T[0, l] and
 * v_cache is T[1, l]. Block b of layer l, plane kv (0 = K, 1 = V) starts at
 *   base + kv * kv_stride + l * layer_stride + b * block_stride
 * and is `chunk_bytes` (= block_size * kv_heads * head_dim * elem_size)
 * contiguous bytes. Strides are signed, so any per-layer (k, v) pair and any
 * affine stack of layers fits this descriptor.
 */
#ifndef LMPOOL_B200_KVX_H
#define LMPOOL_B200_KVX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVX_ABI_VERSION 2

/* ---- host status codes ------------------------------------------------- */
#define KVX_OK 0
#define KVX_EINVAL 1       /* bad argument: ids out of range, duplicate target ids, misaligned layout */
#define KVX_ENOMEM 2       /* device allocation failed (kvx_mailbox_create only) */
#define KVX_ETIMEDOUT 3    /* reserved for host-side waits */
#define KVX_EPEER 4        /* peer access / CUDA IPC failure */
#define KVX_ECUDA 5        /* any other CUDA runtime error */
#define KVX_EUNSUPPORTED 6 /* request outside what this build supports */

/* ---- device status bits (OR-ed into *status_dev by kernels) -------------- */
#define KVX_DEV_BAD_SRC_ID 0x01     /* a source block id was < 0 or >= num_blocks; that chunk skipped */
#define KVX_DEV_BAD_DST_ID 0x02     /* a destination block id was out of range; that chunk skipped */
#define KVX_DEV_BAD_SLOT 0x04       /* a slot_mapping entry was < -1 or >= num_blocks*block_size */
#define KVX_DEV_TIMEOUT 0x08        /* a bounded wait on a peer flag ran out */
#define KVX_DEV_COUNT_MISMATCH 0x10 /* destination posted a different block count than the source moves */
#define KVX_DEV_PEER_FAILED 0x20    /* the peer signalled that its side of the transfer failed */
#define KVX_DEV_PIPE_TIMEOUT 0x40   /* a bounded wait on a bulk-copy barrier ran out */

/* ---- layout descriptor -------------------------------------------------- */
typedef struct kvx_cache_desc {
    uint64_t base;         /* device address of block 0 of layer 0, plane K */
    int64_t kv_stride;     /* bytes from plane K to plane V of the same layer */
    int64_t layer_stride;  /* bytes from layer l to layer l+1 */
    int64_t block_stride;  /* bytes from block b to block b+1 */
    int64_t num_blocks;    /* N: valid block ids are [0, N) */
    int64_t chunk_bytes;   /* contiguous bytes of one (plane, layer, block) */
    int32_t num_layers;    /* L */
    int32_t reserved;      /* must be 0 */
} kvx_cache_desc;

/* Per-rank mailbox: small device region, exported over CUDA IPC, through
 * which a pair agrees on target block ids and completion tokens. */
typedef struct kvx_mailbox {
    uint64_t base;         /* device address (local, or a peer's region mapped by kvx_ipc_open) */
    int32_t max_peers;     /* world size the mailbox was created for */
    int32_t reserved;      /* must be 0 */
    int64_t max_blocks;    /* capacity of each per-peer target-id slot */
} kvx_mailbox;

/* One destination of a push launch (kvx_pair_push). */
typedef struct kvx_push_target {
    kvx_cache_desc dst;            /* destination cache; base is the peer mapping */
    kvx_mailbox dst_mailbox;       /* destination's mailbox, peer mapping */
    const int64_t* src_ids_dev;    /* source block ids (local device memory) */
    int64_t num_ids;               /* blocks to move */
    int32_t dst_rank;              /* destination rank (index into mailboxes) */
    int32_t reserved;              /* must be 0 */
} kvx_push_target;

/* One source of a pull launch (kvx_pair_pull). */
typedef struct kvx_pull_source {
    kvx_cache_desc src;            /* source rank's cache; base is the peer mapping */
    kvx_mailbox src_mailbox;       /* source rank's mailbox, peer mapping */
    const int64_t* src_ids_dev;    /* block ids in the source cache (this GPU's memory) */
    const int64_t* dst_ids_dev;    /* reserved block ids in the local cache (this GPU's memory) */
    int64_t num_ids;               /* blocks to move */
    uint64_t token;                /* signalled to the source when its blocks are read, in [1, 2^63) */
    int32_t src_rank;              /* source rank (index into mailboxes) */
    int32_t reserved;              /* must be 0 */
} kvx_pull_source;

/* Kernel selection knobs (process-wide; for measurement sweeps). */
typedef struct kvx_tuning {
    int32_t variant;       /* 0 = automatic, 1 = register (16-byte ld/st) copy, 2 = TMA bulk copy */
    int32_t ctas_per_sm;   /* 0 = automatic */
    int32_t tile_bytes;    /* 0 = automatic; else multiple of 16 */
    int32_t stages;        /* TMA ring depth; 0 = automatic */
    int32_t store_pdl;     /* store_kvcache launch: 0 = automatic (programmatic dependent launch), 1 = on, 2 = off */
    int32_t reserved;      /* must be 0 */
} kvx_tuning;

/* ---- library ------------------------------------------------------------ */
int kvx_abi_version(void);
const char* kvx_last_error(void);
const char* kvx_status_name(int status);
int kvx_set_tuning(const kvx_tuning* tuning);
int kvx_get_tuning(kvx_tuning* out);

/* Host-only checks (no GPU needed).
 * kvx_validate_block_ids: every id in [0, num_blocks); when require_distinct
 * is non-zero, no id repeats (index_copy_ targets must be distinct:
 * kv_transfer.py:213-215; BlockManager never reserves twice,
 * block_manager.py:521-538). Returns KVX_EINVAL on the first violation. */
int kvx_validate_block_ids(const int64_t* ids, int64_t n, int64_t num_blocks, int32_t require_distinct);
/* *overlap_out = 1 when the two id sets intersect. */
int kvx_ids_overlap(const int64_t* a, int64_t na, const int64_t* b, int64_t nb, int64_t num_blocks,
                    int32_t* overlap_out);
/* Validate a descriptor (alignment, sizes). */
int kvx_check_desc(const kvx_cache_desc* desc);

/* ---- device info -------------------------------------------------------- */
int kvx_device_count(int32_t* out);
int kvx_device_sm_count(int32_t device, int32_t* out);
int kvx_can_access_peer(int32_t device, int32_t peer, int32_t* out);

/* ---- local gather/scatter (kernel 1) -------------------------------------
 * For every plane kv, layer l and i < num_ids copies chunk_bytes from
 *   src block src_ids[i]  to  dst block dst_ids[i].
 * A NULL id pointer means the identity map (id = i), which turns the call
 * into _pack_all_layer_blocks (dst = a payload [L, 2, B, ...] described with
 * block_stride = chunk, kv_stride = B*chunk, layer_stride = 2*B*chunk) or
 * _unpack_all_layer_blocks (src = payload). src and dst may live on this GPU
 * or dst may be a peer mapping. Source and destination chunks must not
 * overlap in memory (callers stage through a payload when they do). */
int kvx_move_blocks(int32_t device, const kvx_cache_desc* src, const kvx_cache_desc* dst,
                    const int64_t* src_ids_dev, const int64_t* dst_ids_dev, int64_t num_ids,
                    int32_t* status_dev, void* stream);

/* ---- pair transfer over NVLink (kernel 2) --------------------------------
 * Replaces kv_transfer.swap_in(negotiate_blocks=False) (kv_transfer.py:395-475).
 * Tokens are issued by the destination, one per transfer, strictly
 * increasing per (source, destination) pair, starting at 1.
 *
 * Destination (execute_swap_in):
 *   kvx_pair_publish   copies its reserved target ids into the source's
 *                      mailbox and release-stores `token` as the arm flag.
 *   kvx_pair_wait_done waits (bounded) until the source's completion flag
 *                      equals `token`; KVX_DEV_TIMEOUT or KVX_DEV_PEER_FAILED
 *                      in *status_dev otherwise.
 * Source (execute_swap_out):
 *   kvx_pair_wait_armed waits (bounded) for an arm token newer than the last
 *                      one consumed from that destination and checks the
 *                      posted id count against num_ids.
 *   kvx_pair_push       one launch moving every target: reads source chunks
 *                      from local HBM and stores them straight into the
 *                      destination's KV cache over NVLink, then its last CTA
 *                      per target release-stores the token into the target's
 *                      completion flag.
 */
int kvx_pair_publish(int32_t device, const kvx_mailbox* src_mailbox_mapped, int32_t my_rank,
                     const int64_t* dst_ids_dev, int64_t num_ids, uint64_t token, void* stream);
int kvx_pair_wait_done(int32_t device, const kvx_mailbox* my_mailbox, int32_t src_rank, uint64_t token,
                       uint64_t timeout_ns, int32_t* status_dev, void* stream);
int kvx_pair_wait_armed(int32_t device, const kvx_mailbox* my_mailbox, const kvx_mailbox* dst_mailbox_mapped,
                        int32_t my_rank, int32_t dst_rank, int64_t num_ids, uint64_t timeout_ns,
                        int32_t* status_dev, void* stream);
int kvx_pair_push(int32_t device, const kvx_cache_desc* src, const kvx_mailbox* my_mailbox, int32_t my_rank,
                  const kvx_push_target* targets, int32_t num_targets, int32_t* status_dev, void* stream);

/* ---- pair transfer, destination-driven (pull) ------------------------------
 * Same replacement of swap_in (kv_transfer.py:395-475), driven by the
 * destination, which already holds both id lists (execute_swap_in receives
 * the source ids and its reserved targets, model_runner.py:777-806). The
 * reference's source packs on its own stream after all earlier work
 * (kv_transfer.py:463-466), so its blocks are read only once the source's
 * own writes to them are done; the grant keeps that ordering:
 *   kvx_pair_request     (destination) posts the block count (tagged as a
 *                        pull) and the arm token into the source's mailbox.
 *   kvx_pair_grant       (source) waits (bounded) for an arm newer than the
 *                        last one consumed from that destination, checks the
 *                        count, and release-stores the token into the
 *                        destination's done[src] flag (token | FAIL on a
 *                        count mismatch). Enqueued on the source's stream, it
 *                        runs after every earlier kernel there, so blocks the
 *                        source was still writing are complete before the
 *                        destination can see the grant.
 *   kvx_pair_wait_done   (destination) waits (bounded) for the grant.
 *   kvx_pair_pull        (destination) one launch reading every source's
 *                        chunks from its cache over NVLink with bulk copies
 *                        and storing them into the local reserved blocks. A
 *                        source's segment copies only if done[src] equals
 *                        that source's token when the launch starts (else it
 *                        copies nothing). The last CTA per source
 *                        release-stores the token (token | FAIL if the
 *                        segment did not copy or a CTA failed) into the
 *                        source's `pulled` flag. The data is in place when
 *                        the launch completes.
 *   kvx_pair_wait_pulled (source, optional) waits (bounded) until the
 *                        destination reports a pull newer than the last one
 *                        consumed and at least as new as the last token this
 *                        rank granted it (a report of an earlier transfer the
 *                        source did not wait for never satisfies a newer
 *                        one); FAIL -> KVX_DEV_PEER_FAILED.
 * A push arm and a pull request never satisfy each other (the count words
 * differ), so two ends that disagree on the mode fail instead of moving data.
 * Measured on B200 at Qwen3-8B geometry, B=64: 777 GB/s per direction for
 * pull against 713 GB/s for push (NVLink reads carry less packet overhead
 * than posted writes). */
int kvx_pair_request(int32_t device, const kvx_mailbox* src_mailbox_mapped, int32_t my_rank, int64_t num_ids,
                     uint64_t token, void* stream);
int kvx_pair_grant(int32_t device, const kvx_mailbox* my_mailbox, const kvx_mailbox* dst_mailbox_mapped,
                   int32_t my_rank, int32_t dst_rank, int64_t num_ids, uint64_t timeout_ns, int32_t* status_dev,
                   void* stream);
int kvx_pair_pull(int32_t device, const kvx_cache_desc* dst, const kvx_mailbox* my_mailbox, int32_t my_rank,
                  const kvx_pull_source* sources, int32_t num_sources, int32_t* status_dev, void* stream);
int kvx_pair_wait_pulled(int32_t device, const kvx_mailbox* my_mailbox, int32_t dst_rank, uint64_t timeout_ns,
                         int32_t* status_dev, void* stream);

/* ---- allocation-free push ---------------------------------------------------
 * No counterpart in the reference: LMPool has no such entry point.
 *
 * Some callers cannot call cudaMalloc: a serving process whose memory is
 * already handed out (LMPool sizes its KV cache to take the configured share
 * of all free GPU memory), a plugin whose host program forbids it to
 * allocate device memory, or a host whose own allocator owns every byte of
 * device memory.
 * kvx_pair_push keeps its scratch -- one CTA-completion counter per
 * destination rank -- in the mailbox region, which kvx_mailbox_create
 * allocates with cudaMalloc. This variant moves the same bytes with the same
 * kernel, results identical to kvx_pair_push, but keeps those counters in a
 * fixed array inside this library (KVX_NOALLOC_MAX_PEERS counters, 256
 * bytes, held by every GPU that loads the library until the process exits),
 * so it allocates nothing and needs no scratch from the caller. The caller
 * still passes its inputs and outputs (caches, source ids, and a mailbox
 * placed in memory it owns: any zeroed region of kvx_mailbox_bytes() bytes).
 *   - Destination ranks must be < KVX_NOALLOC_MAX_PEERS; larger ranks are
 *     rejected with KVX_EINVAL.
 *   - The first call on a device resolves the array's device address
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *   - Every call shares the array, one counter per destination rank. Each
 *     call clears its destinations' counters on `stream` before launching,
 *     so any two calls on the same device whose pushes to one destination
 *     rank overlap on the GPU race and must not be issued: two streams of one
 *     caller, or two callers acting as different source ranks on one GPU.
 */
#define KVX_NOALLOC_MAX_PEERS 64
int kvx_pair_push_noalloc(int32_t device, const kvx_cache_desc* src, const kvx_mailbox* my_mailbox,
                          int32_t my_rank, const kvx_push_target* targets, int32_t num_targets,
                          int32_t* status_dev, void* stream);

/* ---- mailbox and CUDA IPC (replaces pair communicators) -------------------
 * kvx_mailbox_create allocates and zeroes a mailbox on `device`
 * (kv_transfer.py:64-71 created a pair NCCL group instead). */
int kvx_mailbox_bytes(int32_t max_peers, int64_t max_blocks, uint64_t* bytes_out);
int kvx_mailbox_create(int32_t device, int32_t max_peers, int64_t max_blocks, kvx_mailbox* out);
int kvx_mailbox_destroy(int32_t device, const kvx_mailbox* mailbox);
/* Last completion token this rank received from `src_rank` (host read). */
int kvx_mailbox_read_done(int32_t device, const kvx_mailbox* mailbox, int32_t src_rank, uint64_t* token_out);
/* Zero every word of `peer`'s pair state in this rank's own mailbox (arm,
 * count, done, consumed, go, pulled, granted and both CTA counters), enqueued on
 * `stream`. Both ranks of a pair call it, with no transfer of that pair in
 * flight, before they start again from token 1: how a pair disabled after a
 * timeout is brought back without recreating the mailbox (prewarm does it). */
int kvx_mailbox_reset_peer(int32_t device, const kvx_mailbox* mailbox, int32_t peer, void* stream);

/* Export the allocation holding dev_ptr: 64-byte cudaIpcMemHandle_t plus the
 * byte offset of dev_ptr inside that allocation. */
int kvx_ipc_export(int32_t device, const void* dev_ptr, void* handle_out_64, uint64_t* offset_out);
/* Map a peer allocation into this process on `device`; returns base+offset. */
int kvx_ipc_open(int32_t device, const void* handle_64, uint64_t offset, uint64_t* ptr_out);
int kvx_ipc_close(int32_t device, uint64_t ptr, uint64_t offset);
/* Same-process peers (one process driving several GPUs): enable access. */
int kvx_enable_peer_access(int32_t device, int32_t peer);

/* ---- store_kvcache (kernel 3) ---------------------------------------------
 * Replaces layers/attention.py:67-108 (Triton kernel :7-64). For each token
 * t < num_tokens with slot = slot_mapping[t] != -1:
 *   k_cache[slot / block_size, slot % block_size, :, :] = key[t, :, :]
 *   v_cache[...]                                         = value[t, :, :]
 * key/value rows (kv_heads*head_dim elements, `row_bytes` bytes) are
 * contiguous; token stride may differ from row_bytes. Cache rows are
 * addressed as block * cache_block_stride + (slot % block_size) * cache_slot_stride.
 * Slots outside [-1, num_blocks*block_size) are skipped and flagged with
 * KVX_DEV_BAD_SLOT. No allocation, no host synchronisation: safe inside CUDA
 * graph capture. */
int kvx_store_kvcache(int32_t device, const void* key_dev, const void* value_dev, int64_t key_token_stride,
                      int64_t value_token_stride, void* k_cache_dev, void* v_cache_dev, int64_t cache_block_stride,
                      int64_t cache_slot_stride, const int64_t* slot_mapping_dev, int64_t num_tokens,
                      int64_t num_blocks, int32_t block_size, int64_t row_bytes, int32_t* status_dev, void* stream);
/* All layers in one launch: layer l adds l * *_layer_stride to key, value,
 * k_cache and v_cache; one slot_mapping serves every layer (it is per token,
 * utils/context.py). */
int kvx_store_kvcache_layers(int32_t device, int32_t num_layers, const void* key_dev, const void* value_dev,
                             int64_t key_layer_stride, int64_t value_layer_stride, int64_t key_token_stride,
                             int64_t value_token_stride, void* k_cache_dev, void* v_cache_dev,
                             int64_t k_cache_layer_stride, int64_t v_cache_layer_stride, int64_t cache_block_stride,
                             int64_t cache_slot_stride, const int64_t* slot_mapping_dev, int64_t num_tokens,
                             int64_t num_blocks, int32_t block_size, int64_t row_bytes, int32_t* status_dev,
                             void* stream);

/* ---- bounded waits for tests of the failure path -------------------------
 * Waits on *flag_dev >= expected with a timeout; ORs KVX_DEV_TIMEOUT into
 * *status_dev when it runs out. Never traps, never hangs past the bound. */
int kvx_wait_flag(int32_t device, const uint64_t* flag_dev, uint64_t expected, uint64_t timeout_ns,
                  int32_t* status_dev, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LMPOOL_B200_KVX_H */
