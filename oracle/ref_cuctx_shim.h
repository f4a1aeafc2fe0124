/* Force-included when compiling the reference harness (QuickRunCUDA.cpp) with
 * CUDA 12.9.  The harness calls cuCtxCreate(&ctx, NULL, 0, dev)
 * (QuickRunCUDA.cpp:287), the CUDA 13 signature; in CUDA 12.9 cuda.h maps the
 * name to the 3-argument cuCtxCreate_v2, while the same 4-argument entry point
 * is exported as cuCtxCreate_v4.  With a NULL parameter block both create a
 * plain context on the device. */
#include <cuda.h>
#undef cuCtxCreate
#define cuCtxCreate cuCtxCreate_v4
