// qrc_noalloc.cu -- qrc_absmax_f32_noalloc: the side-aware absmax for callers
// that cannot allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is not allowed or not wanted.
// Examples are a host application that reserves all device memory up front
// and hands its plugins only the buffers they work on, a serving process held
// to a fixed memory budget, and code that must not trigger the implicit
// synchronisation cudaMalloc may cause.  Such a caller passes its input and
// output buffers and nothing else; the scratch this reduction needs (side map,
// work queues, ticket, accumulator) lives in the fixed array below, which every
// GPU that loads this library holds until the process exits.
//
// This is the same reduction as qrc_absmax_f32 (side_aware_b200.cu), run on a
// statically allocated map instead of a context's.
#define QRC_NO_PLUGIN_ABI
#include "side_aware_b200.cu"
#include "../../include/qrc_b200.h"

#include <cuda_runtime.h>
#include <mutex>

#define QRC_API extern "C" __attribute__((visibility("default")))

namespace {

// Scratch size: the map header plus one bit per 2 MiB page for up to 32768
// pages, i.e. inputs spanning at most 64 GiB.  20 KiB per device.
constexpr size_t kNoallocPageWords = qrc::kDefaultPageWords;
constexpr size_t kNoallocWords = qrc::O_PAGE_BITS + kNoallocPageWords;
constexpr uint64_t kNoallocMaxPages = (uint64_t)kNoallocPageWords * 32;

// Per-device state: the device address of the scratch array (found once per
// device with cudaGetSymbolAddress) and the input range its side map describes.
// The address belongs to the device's primary context as it was at set-up:
// after cudaDeviceReset the entry point must not be used again in the same
// process (the array would be a different allocation).
struct NoallocDevice {
    bool ready = false;
    qrc_u32* scratch = nullptr;
    int num_sms = 0;
    uint64_t mapped_base = 0, mapped_bytes = 0;
};
constexpr int kMaxDevices = 64;
NoallocDevice g_devices[kMaxDevices];
std::mutex g_mutex;

}  // namespace

static __device__ __align__(256) qrc_u32 g_noalloc_scratch[kNoallocWords];

__global__ void __launch_bounds__(1024, 1)
qrc_k_noalloc_discover(const void* base, qrc_u64 bytes, qrc_u32* map) {
    qrc::discover(base, bytes, map);
}

__global__ void __launch_bounds__(1024, 1)
qrc_k_noalloc_absmax_f32(const float* in, qrc_u64 n, qrc_u32* map, float* out) {
    qrc::reduce_run<qrc::OpAbsF32>(in, n, map, out, nullptr, qrc::MODE_SIDE_AWARE);
}

#define QRC_NA_CK(call)                                       \
    do {                                                      \
        if ((call) != cudaSuccess) return QRC_ERR_CUDA;       \
    } while (0)

QRC_API int qrc_absmax_f32_noalloc(const float* d_in, size_t n, float* d_out, void* stream) {
    if (!d_out || (n && !d_in) || ((uintptr_t)d_in & 3)) return QRC_ERR_INVALID;
    const uint64_t a = (uintptr_t)d_in, bytes = (uint64_t)n * 4;
    const uint64_t pages = n ? (a + bytes + qrc::kPage - 1) / qrc::kPage - a / qrc::kPage : 0;
    if (n > ((size_t)1 << 61) || pages > kNoallocMaxPages) return QRC_ERR_RANGE;

    int dev = 0;
    QRC_NA_CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return QRC_ERR_DEVICE;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

    std::lock_guard<std::mutex> lock(g_mutex);
    NoallocDevice& d = g_devices[dev];
    if (!d.ready) {
        // Set-up, once per device, with that device current: the host-side
        // name g_noalloc_scratch is not a device address; ask for the real one.
        int major = 0;
        QRC_NA_CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
        if (major != 10) return QRC_ERR_DEVICE;
        QRC_NA_CK(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev));
        void* ptr = nullptr;
        QRC_NA_CK(cudaGetSymbolAddress(&ptr, g_noalloc_scratch));
        d.scratch = static_cast<qrc_u32*>(ptr);
        d.mapped_base = d.mapped_bytes = 0;
        d.ready = true;
    }
    if (d.mapped_base != a || d.mapped_bytes != bytes) {
        // New input range: clear the whole array (map, queues, ticket and
        // accumulator must start at zero) and rediscover for this range.
        // The range is recorded only once both are queued, so a failure here
        // makes the next call start over instead of trusting a cleared map.
        d.mapped_base = d.mapped_bytes = 0;
        QRC_NA_CK(cudaMemsetAsync(d.scratch, 0, kNoallocWords * sizeof(qrc_u32), s));
        if (n) qrc_k_noalloc_discover<<<d.num_sms, 1024, 0, s>>>(d_in, bytes, d.scratch);
        QRC_NA_CK(cudaGetLastError());
        d.mapped_base = a;
        d.mapped_bytes = bytes;
    }
    // Queues, ticket and accumulator are back at zero after every completed
    // launch (the last CTA resets them), so the next call starts clean.
    qrc_k_noalloc_absmax_f32<<<d.num_sms, 1024, 0, s>>>(d_in, (qrc_u64)n, d.scratch, d_out);
    QRC_NA_CK(cudaGetLastError());
    return QRC_OK;
}
