/*
 * qrc_b200.h -- C ABI of the B200-native side-aware absmax library
 * (libqrc_b200.so).
 *
 * The reference (QuickRunCUDA) exposes this path only through its kernel-file
 * plugin ABI: the harness allocates A/B/C, launches `init` once and `kernel`
 * T times, and reads C[0] (QuickRunCUDA.cpp:354-658, tests/side_aware.cu:72,
 * :257).  The library keeps that ABI (quickruncuda_b200/csrc/side_aware_b200.cu
 * is a drop-in kernel file) and adds these plain-C entry points so host C/C++
 * code can call the same reduction directly.  Each entry point names the
 * reference interface it replaces.
 *
 * Conventions
 *   - All pointers named d_* are device pointers owned by the caller; h_* are
 *     host pointers.  No function takes or returns a torch or CUDA C++ type:
 *     streams are passed as `void*` holding a cudaStream_t (NULL = legacy
 *     default stream).
 *   - Every function returns QRC_OK (0) or a negative qrc_status.
 *   - Reductions are asynchronous on the given stream unless stated.
 *   - A context owns device scratch (the side map, its work queues and the
 *     accumulator): at most one reduction per context may be in flight at a
 *     time; use one context per stream or thread.
 */
#ifndef QRC_B200_H
#define QRC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct qrc_ctx qrc_ctx;

enum qrc_status {
    QRC_OK = 0,
    QRC_ERR_INVALID = -1,   /* bad argument (NULL pointer, size, alignment) */
    QRC_ERR_CUDA = -2,      /* a CUDA runtime call failed; see qrc_last_cuda_error() */
    QRC_ERR_DEVICE = -3,    /* no such device, or not an sm_100 device */
    QRC_ERR_RANGE = -4,     /* input too large for this entry point */
    QRC_ERR_STATE = -5      /* context used with a different device */
};

/* Read modes.  SIDE_AWARE is the product path; the others exist for the
 * ablations of the reference (tests/side_aware.cu:19-20, :305-311). */
enum qrc_mode {
    QRC_MODE_SIDE_AWARE = 0,        /* each side reads the chunks homed on it */
    QRC_MODE_IGNORE_PAGE_BITS = 1,  /* FORCE_RANDOM_SIDE: page bits treated as 0 */
    QRC_MODE_WRONG_SIDE = 2,        /* FORCE_WRONG_SIDE: every chunk read across the die boundary */
    QRC_MODE_STREAM = 3,            /* plain grid-stride stream, no side logic */
    /* Work schedule, OR-ed into a side-aware mode (default: chosen by size). */
    QRC_SCHED_STATIC = 0x10,        /* every SM reads a fixed share: no atomics */
    QRC_SCHED_QUEUE = 0x20,         /* warps take one-pair grabs from per-side queues */
    QRC_SCHED_BALANCED = 0x30       /* static shares for 5/8 of the input (1/8 above
                                       1 GiB), the rest claimed in 64 KiB blocks from
                                       per-side queues */
};

/* Discovery status (qrc_side_info.status). */
enum qrc_side_status {
    QRC_SIDE_OK = 0,
    QRC_SIDE_TOO_SMALL = 1,         /* no full 2 MiB page inside the buffer */
    QRC_SIDE_NO_SM_SPLIT = 2,       /* SM latencies did not form two clusters */
    QRC_SIDE_NO_HASH = 3,           /* no address bit 4..20 changed the side */
    QRC_SIDE_BAD_HASH = 4,          /* lowest hash bit below 512 bytes */
    QRC_SIDE_NO_CAL_SPLIT = 5,      /* calibration words not separable */
    QRC_SIDE_VERIFY_FAILED = 6,     /* map mispredicted > 1/8 of verification probes */
    QRC_SIDE_TOO_MANY_PAGES = 7,    /* more pages than the map can hold */
    QRC_SIDE_UNALIGNED = 8,         /* base not 4-byte aligned */
    QRC_SIDE_NOT_RUN = 100          /* context created without a buffer */
};

typedef struct qrc_side_info {
    uint32_t status;            /* qrc_side_status */
    uint32_t mask;              /* in-page side hash mask in use (0 when not side-aware) */
    uint32_t mask_measured;     /* mask as measured, even when rejected */
    uint32_t chunk_bytes;       /* lowest hash bit: bytes per side chunk */
    uint32_t num_sms_measured;
    uint32_t sms_side0;
    uint32_t sms_side1;
    uint32_t num_pages;         /* 2 MiB pages spanned by the buffer */
    uint32_t verify_probes;
    uint32_t verify_mismatches;
    uint32_t cal_lat_side0;     /* cycles for 32 dependent atomics, discovering SM -> side 0 word */
    uint32_t cal_lat_side1;     /* same, side 1 word */
    uint32_t sm_lat_cluster0;   /* phase-1 cluster means (cycles per 32 atomics) */
    uint32_t sm_lat_cluster1;
    uint32_t discover_smid;     /* SM that ran phase 2 */
    uint32_t reserved;
} qrc_side_info;

/* Create a context for `device` and, when d_base != NULL, run side discovery
 * on the device allocation [d_base, d_base + bytes): SM sides, the in-page
 * hash mask and one side bit per 2 MiB page.  Synchronous (returns after the
 * discovery kernel finished on `stream`).  Discovery reads the buffer with
 * same-value atomics and never changes its contents, but no other work may
 * write that memory while it runs.  d_base == NULL creates a context without
 * a map: reductions then run side-agnostic.
 * Replaces: the harness' `-i` init launch on (A, B) -- QuickRunCUDA.cpp:477-487
 * calling tests/side_aware.cu:72 `init`. */
int qrc_ctx_create(qrc_ctx** out, int device, const void* d_base, size_t bytes, void* stream);

/* Free a context and its device scratch.  NULL is accepted. */
int qrc_ctx_destroy(qrc_ctx* ctx);

/* Copy the discovery result.  Replaces the init kernel's debug printout
 * (tests/side_aware.cu:95-197). */
int qrc_ctx_get_info(const qrc_ctx* ctx, qrc_side_info* info);

/* Select the read mode (qrc_mode, optionally OR-ed with a QRC_SCHED_* bit)
 * for later reductions on this context.
 * Replaces the compile-time FORCE_RANDOM_SIDE / FORCE_WRONG_SIDE defines
 * (tests/side_aware.cu:19-20). */
int qrc_ctx_set_mode(qrc_ctx* ctx, int mode);

/* Launch shape for later reductions: blocks per SM (1 or 2) and threads per
 * block (256, 512 or 1024; blocks_per_sm * threads <= 2048).  Default 1 x 1024,
 * the reference's `-p -t 1024` (QuickRunCUDA.cpp:365-369). */
int qrc_ctx_set_launch(qrc_ctx* ctx, int blocks_per_sm, int threads_per_block);

/* Load pipeline for later reductions.  0 (default): each warp keeps eight
 * 16-byte loads per lane in flight in registers (128 KiB per SM at 1024
 * threads).  2..16: each warp stages its chunks through that many 4 KiB
 * shared-memory slots filled by 1-D bulk async copies (cp.async.bulk with
 * mbarrier completion), so up to threads/32 * slots * 4 KiB per SM are in
 * flight without registers; needs blocks_per_sm == 1 and
 * threads/32 * slots * 4104 <= 227 KiB (e.g. 256 threads x 6 slots).
 * No reference counterpart (the reference uses register loads only,
 * tests/side_aware.cu:319-325). */
int qrc_ctx_set_pipeline(qrc_ctx* ctx, int bulk_slots_per_warp);

/* Programmatic dependent launch of reductions (1, the default) or plain
 * stream order (0).  With 1, a reduction's CTAs may be scheduled while the
 * previous kernel in the stream drains; each reduction still waits for that
 * kernel to complete before it uses any memory (griddepcontrol.wait), so
 * results and ordering are unchanged and only launch latency is hidden.
 * No reference counterpart (the harness launches with cuLaunchKernel,
 * QuickRunCUDA.cpp:528-532). */
int qrc_ctx_set_overlap(qrc_ctx* ctx, int enable);

/* *d_out = max_i |d_in[i]| over n floats (IEEE maxNum: NaN inputs are ignored,
 * -0 gives +0, n == 0 gives +0).  d_in must be 4-byte aligned; the side-aware
 * path applies when [d_in, d_in + n) lies inside the context's buffer.
 * Bit-exact and deterministic.  Asynchronous on `stream`.
 * Replaces: one timed launch of `kernel` (QuickRunCUDA.cpp:528-532 ->
 * tests/side_aware.cu:257-395) with C[0] as the output. */
int qrc_absmax_f32(const float* d_in, size_t n, float* d_out, qrc_ctx* ctx, void* stream);

/* Reduction operators of qrc_reduce_f32. */
enum qrc_op {
    QRC_OP_ABSMAX = 0,              /* max |x|, float result (as qrc_absmax_f32) */
    QRC_OP_MAX = 1,                 /* max x, float; NaN skipped, -0 below +0, empty gives -inf */
    QRC_OP_MIN = 2,                 /* min x, float; NaN skipped, -0 below +0, empty gives +inf */
    QRC_OP_SUM = 3,                 /* sum of x in double, double result */
    QRC_OP_SUMSQ = 4                /* sum of x*x in double, double result */
};

/* The same side-aware walk with another reduction operator.  *d_out is one
 * float for ABSMAX/MAX/MIN (bit-exact, deterministic) and one double for
 * SUM/SUMSQ (d_out 8-byte aligned; every element is added exactly once, in
 * an order that varies between launches, so the last bits may differ from
 * one launch to the next).  Same context, alignment and stream rules as
 * qrc_absmax_f32.
 * Replaces: the reference's swappable reduction operator
 * (tests/side_aware.cu:215-219), which needs an edit and a recompile there. */
int qrc_reduce_f32(const float* d_in, size_t n, int op, void* d_out, qrc_ctx* ctx, void* stream);

/* Same reduction for callers that cannot allocate device memory: a host
 * application that reserves all device memory up front and hands this code
 * only the buffers it works on, a process held to a fixed memory budget, or
 * code that must avoid the implicit synchronisation cudaMalloc may cause.
 * Neither this call nor anything it calls allocates: no context is needed,
 * and its scratch (side map, work queues, ticket, accumulator; 20 KiB) is a
 * fixed array that every GPU loading this library holds until exit.  Runs on
 * the current device, asynchronously on `stream`.
 *   - Limit: the input may span at most 32768 pages of 2 MiB (64 GiB, about
 *     16e9 floats); larger inputs return QRC_ERR_RANGE before any GPU work.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress); make it before any stream capture.
 *   - The array remembers the last input range: a call on a new range clears
 *     it and runs side discovery for that range first (about 1-2 ms for 4 GB);
 *     repeated calls on the same buffer reuse the map.
 *   - Every call on a device shares the one array, so calls that overlap on
 *     the GPU (other streams, other host threads) race; serialise them.
 *   - The array's address is looked up once per device; do not call this
 *     entry point again after cudaDeviceReset in the same process.
 * Result and errors as qrc_absmax_f32.  No counterpart in the reference. */
int qrc_absmax_f32_noalloc(const float* d_in, size_t n, float* d_out, void* stream);

/* Same result from a host buffer: copies h_in to a device staging buffer owned
 * by the context in 256 MiB chunks on the context's own copy stream, reduces
 * each chunk on `stream` as soon as it has landed (so the reductions hide
 * under the copies), takes the maximum of the chunk results on the device and
 * copies it to *h_out.  The copies start after the work queued on `stream`
 * before the call.  Synchronous.  Pinned host memory gives full PCIe
 * bandwidth.  The staging is set up by the first call that needs it (or by
 * qrc_host_reserve) and kept by the context.
 * Replaces: the harness' fill-and-copy of A (QuickRunCUDA.cpp:432-457) followed
 * by a kernel launch and the C dump (:594-615). */
int qrc_absmax_f32_host(const float* h_in, size_t n, float* h_out, qrc_ctx* ctx, void* stream);

/* Sets up the staging of qrc_absmax_f32_host for inputs of up to n floats
 * ahead of time: a device buffer of n floats with its own side map
 * (discovery runs on it, synchronously), a copy stream, one event and one
 * partial-result float per 256 MiB chunk.  A larger n replaces the staging; a
 * smaller one keeps it.  On failure nothing is kept and the next call retries.
 * Replaces: the harness' allocation of A before its first launch
 * (QuickRunCUDA.cpp:360-362). */
int qrc_host_reserve(qrc_ctx* ctx, size_t n);

/* Fused per-tensor FP8 quantize of n bf16 values (raw bit patterns):
 *   amax = max |x| (maxNum), *d_scale = 448 / amax (IEEE division; 1 when amax
 *   is 0 or infinite), d_q[i] = e4m3(x[i] * scale) with round-to-nearest-even
 *   and saturation to +-448 (OCP OFP8 E4M3).  d_amax (may be NULL) receives
 *   amax.  Asynchronous.  When d_in_bf16 lies inside the context's
 *   side-aware buffer (16-byte aligned, d_q 8-byte aligned) and discovery
 *   labelled every SM, this is one launch of one CTA per SM: the amax pass
 *   keeps its last blocks in tensor and shared memory across a bounded grid
 *   barrier, then quantizes; otherwise two launches (amax, then quantize).
 *   Both give the same bytes.  If the one-launch path's barrier wait gives up
 *   (about 1 s), amax is NaN and scale 1, and d_q holds no valid result.
 *   No reference counterpart: the quantize extends the reduction of
 *   tests/side_aware.cu:216-219 to the quant_infer use case. */
int qrc_amax_quant_e4m3(const uint16_t* d_in_bf16, size_t n, uint8_t* d_q, float* d_scale,
                        float* d_amax, qrc_ctx* ctx, void* stream);

/* Sharded absmax with the cross-GPU maximum taken inside the kernel: one
 * process (rank) per GPU, each reducing its own shard.  The last CTA of each
 * rank stores its partial maximum in a slot of every rank's exchange array
 * over NVLink, then waits (bounded, about 2 s) until its own array holds this
 * launch's value from every rank, and writes the maximum over all ranks.
 * Set-up, once per process:
 *   qrc_xchg_create(&x, device, rank, world);
 *   qrc_xchg_get_handle(x, h)          -> send h (QRC_XCHG_HANDLE_BYTES) to every rank;
 *   qrc_xchg_set_peer(x, peer, h_peer) for every other rank (CUDA IPC, so
 *                                         each rank is a separate process).
 * Every rank must then call qrc_absmax_f32_allreduce the same number of times,
 * in the same order, like a collective.  If a peer's value does not arrive in
 * time (a rank died, or calls out of step), *d_out is NaN and the map word
 * H_XCHG_ERR is set; the context stays usable.
 * Replaces: a per-GPU qrc_absmax_f32 followed by an NCCL max all-reduce of one
 * float; the reference has no multi-GPU path (QuickRunCUDA.cpp:286 uses
 * device 0 only). */
#define QRC_XCHG_MAX_WORLD 64
#define QRC_XCHG_HANDLE_BYTES 64
typedef struct qrc_xchg qrc_xchg;
int qrc_xchg_create(qrc_xchg** out, int device, int rank, int world);
int qrc_xchg_get_handle(const qrc_xchg* x, void* handle_out);
int qrc_xchg_set_peer(qrc_xchg* x, int peer, const void* handle);
int qrc_xchg_destroy(qrc_xchg* x);
int qrc_absmax_f32_allreduce(const float* d_in, size_t n, float* d_out, qrc_ctx* ctx, qrc_xchg* x, void* stream);

/* Device memory homed like a context's buffer: *d_ptr points to ctx's buffer
 * size of new memory at the same offset within its first 2 MiB page, built
 * from physical 2 MiB pages chosen (by a discovery run over candidate pages)
 * so that every offset lands on the same die as in the context's buffer.
 * Element-wise work that reads x on its die can then write y there too.
 * Allocates through the driver's virtual memory management (cuMemCreate /
 * cuMemMap).  Candidate pages are created and classified in rounds; while
 * it runs it holds, besides the pages it keeps (the buffer size), one round's
 * candidates: twice the pages still missing plus 4, at most 8192 pages
 * (16 GiB).  Synchronous.
 * Free with qrc_free_like once no work uses the memory.
 * Replaces: nothing in the reference; its README (README.md:14) notes that
 * side-aware element-wise output needs this allocator-level page control. */
typedef struct qrc_vmm_buf qrc_vmm_buf;
int qrc_alloc_like(qrc_vmm_buf** out, void** d_ptr, const qrc_ctx* like);
int qrc_free_like(qrc_vmm_buf* buf);

/* d_y[i] = d_x[i] for n floats.  When d_x lies in ctx's buffer (16-byte
 * aligned, d_y too) each die copies the chunks homed on it; with d_y from
 * qrc_alloc_like the stores stay on the die as well.  Other cases use
 * cudaMemcpyAsync.  Ranges that partly overlap return QRC_ERR_INVALID;
 * d_x == d_y does nothing.  Asynchronous.  No reference counterpart. */
int qrc_copy_f32(const float* d_x, float* d_y, size_t n, qrc_ctx* ctx, void* stream);

/* Synthetic inputs generated on the device; element i of the stream is a pure
 * function of (seed, offset + i), so shards of one stream can be generated
 * independently.  uniform[-1,1) on a 2^-23 grid; normal(0, sigma) is the
 * Irwin-Hall sum of twelve 24-bit uniforms (sigma a power of two keeps it
 * bit-reproducible).  The host variants produce identical bits.
 * No reference counterpart: the harness fills A with masked mt19937_64 bits or
 * zeros only (QuickRunCUDA.cpp:432-463). */
int qrc_fill_uniform_f32(float* d_out, size_t n, uint64_t seed, uint64_t offset, void* stream);
int qrc_fill_normal_f32(float* d_out, size_t n, uint64_t seed, uint64_t offset, float sigma, void* stream);
int qrc_fill_normal_bf16(uint16_t* d_out, size_t n, uint64_t seed, uint64_t offset, float sigma, void* stream);
int qrc_host_fill_uniform_f32(float* h_out, size_t n, uint64_t seed, uint64_t offset);
int qrc_host_fill_normal_f32(float* h_out, size_t n, uint64_t seed, uint64_t offset, float sigma);

/* Seeded outlier placement used by the synthetic workloads: index in [0, n)
 * and sign (+1 / -1). */
uint64_t qrc_outlier_index(uint64_t seed, uint64_t n);
int qrc_outlier_sign(uint64_t seed);

/* Human-readable names. */
const char* qrc_status_string(int status);
const char* qrc_side_status_string(uint32_t side_status);

/* Last CUDA runtime error code seen by the library on this thread (0 = none). */
int qrc_last_cuda_error(void);

/* Library version (major * 10000 + minor * 100 + patch). */
int qrc_version(void);

#ifdef __cplusplus
}
#endif

#endif /* QRC_B200_H */
