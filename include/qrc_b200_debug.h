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

/* Device pointer of the context's side map (for launching the plugin kernels
 * from a test on the same scratch). */
void* qrc_ctx_map_device_ptr(const struct qrc_ctx* ctx);

#ifdef __cplusplus
}
#endif

#endif /* QRC_B200_DEBUG_H */
