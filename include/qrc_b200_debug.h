/*
 * qrc_b200_debug.h -- diagnostic entry points of libqrc_b200.so, used by the
 * test suite and by people inspecting discovery.  Not needed on the data path.
 * No reference counterpart: the reference prints its discovery state from the
 * init kernel (tests/side_aware.cu:95-197) instead.
 */
#ifndef QRC_B200_DEBUG_H
#define QRC_B200_DEBUG_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct qrc_ctx;

/* Copy the first `words` 32-bit words of the context's side map (the same
 * layout the plugin kernel file keeps in buffer B) to host memory.
 * Synchronous.  Returns the number of words the map holds through *total. */
int qrc_ctx_read_map(const struct qrc_ctx* ctx, uint32_t* h_words, size_t words, size_t* total);

/* Zero the map's error and coverage words (used with the checked build, which
 * records the first out-of-range access and the bytes / address hash of every
 * access).  Synchronous. */
int qrc_ctx_clear_diagnostics(struct qrc_ctx* ctx);

/* 1 when this library was built with per-access bounds and coverage checks. */
int qrc_is_checked_build(void);

/* d_out[i] = e4m3 code of d_in[i] through the same `cvt.rn.satfinite.e4m3x2`
 * conversion the quantize kernel uses (for an exhaustive comparison against
 * an encoder written from the OCP OFP8 specification).  Asynchronous. */
int qrc_debug_cvt_e4m3(const float* d_in, size_t n, uint8_t* d_out, void* stream);

/* Plain streaming read of bytes [d_in, d_in + bytes) (16-byte aligned; a tail
 * below 16 bytes is skipped) with no side logic, XOR-folded into *d_sink: a
 * measured read-only ceiling for the roofline.  `depth` 16-byte loads in
 * flight per thread; the shapes offered are (depth, threads, blocks per SM) =
 * (8, 1024, 1), (4, 1024, 2), (16, 512, 1) and (32, 256, 1), all 128 KiB in
 * flight per SM.  Runs on the current device.  Asynchronous. */
int qrc_debug_read_stream(const void* d_in, size_t bytes, int depth, int threads, int blocks_per_sm,
                          uint32_t* d_sink, void* stream);

/* Device pointer of the context's side map (for launching the plugin kernels
 * from a test on the same scratch). */
void* qrc_ctx_map_device_ptr(const struct qrc_ctx* ctx);

/* 1 (default): the quantize's second pass reads side-aware when the input is
 * inside the context's mapped buffer and aligned; 0: always the side-agnostic
 * pass (for comparing the two). */
int qrc_ctx_debug_quant_side_aware(struct qrc_ctx* ctx, int enable);

/* 1 (default): qrc_amax_quant_e4m3 runs the single-launch fused kernel
 * whenever its conditions hold (input inside the context's side-aware
 * buffer, 16-byte aligned input, 8-byte aligned output, every SM labelled by
 * discovery, exactly one 1024-thread CTA fits per SM); 0: always the two
 * launches (amax pass, then quantize pass), for comparing the two. */
int qrc_ctx_debug_quant_fused(struct qrc_ctx* ctx, int enable);

/* Kernel launches qrc_amax_quant_e4m3 would make for these arguments: 1 (the
 * fused kernel, or n == 0) or 2. */
int qrc_debug_quant_launches(struct qrc_ctx* ctx, const uint16_t* d_in, size_t n, const uint8_t* d_q);

/* Exchange tests on one GPU: map a peer's slot array to a local device buffer
 * (no IPC), read this rank's slot array, and the epoch of the last launch.
 * With them a test can play a peer from the host (write its slot before the
 * launch) or leave a slot empty and check that the bounded wait gives up. */
struct qrc_xchg;
int qrc_xchg_debug_set_peer_ptr(struct qrc_xchg* x, int peer, void* d_slots);
/* Write (epoch, value) into this rank's slot for `peer`, as that peer would.
 * Synchronous. */
int qrc_xchg_debug_post(struct qrc_xchg* x, int peer, uint32_t epoch, uint32_t value_bits);
void* qrc_xchg_debug_slots(const struct qrc_xchg* x);
uint32_t qrc_xchg_epoch(const struct qrc_xchg* x);

#ifdef __cplusplus
}
#endif

#endif /* QRC_B200_DEBUG_H */
