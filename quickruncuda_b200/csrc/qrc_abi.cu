// qrc_abi.cu -- libqrc_b200.so: the C ABI declared in include/qrc_b200.h.
//
// The device code is the plugin kernel file itself (side_aware_b200.cu, with
// its `init`/`kernel` wrappers compiled out); this file adds kernels with
// launch shapes chosen by the library, the FP8 quantize pass, the synthetic
// generators and the host-side context that owns the side map.
#define QRC_NO_PLUGIN_ABI
#include "side_aware_b200.cu"
#include "qrc_gen.cuh"
#include "../../include/qrc_b200.h"
#include "../../include/qrc_b200_debug.h"

#include <cuda.h>                 // driver types only: entry points come from cudaGetDriverEntryPoint
#include <cuda_runtime.h>
#include <cstring>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>
#include <vector>
#include <omp.h>

#define QRC_API extern "C" __attribute__((visibility("default")))

// ---------------------------------------------------------------------------
// Kernels
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(1024, 1)
qrc_k_discover(const void* base, qrc_u64 bytes, qrc_u32* map) {
    qrc::discover(base, bytes, map);
}

// 64 registers per thread at every shape: 1024 x 1, 512 x 2, 256 x 4 per SM.
template <int T>
__global__ void __launch_bounds__(T, 1024 / T)
qrc_k_absmax_f32(const float* in, qrc_u64 n, qrc_u32* map, float* out, qrc_u32 mode) {
    qrc::reduce_run<qrc::OpAbsF32>(in, n, map, out, nullptr, mode);
}

// absmax whose last CTA also combines with the other GPUs (qrc_xchg).
template <int T>
__global__ void __launch_bounds__(T, 1024 / T)
qrc_k_absmax_f32_xchg(const float* in, qrc_u64 n, qrc_u32* map, float* out, qrc_u32 mode, qrc::XchgArgs xa) {
    qrc::reduce_run<qrc::OpAbsF32>(in, n, map, out, nullptr, mode, xa);
}

// The other operators of qrc_reduce_f32 (absmax keeps its own kernel name).
template <class Op, int T>
__global__ void __launch_bounds__(T, 1024 / T)
qrc_k_reduce_f32(const float* in, qrc_u64 n, qrc_u32* map, void* out, qrc_u32 mode) {
    qrc::reduce_run<Op>(in, n, map, out, nullptr, mode);
}

template <int T>
__global__ void __launch_bounds__(T, 1024 / T)
qrc_k_amax_bf16(const uint16_t* in, qrc_u64 n, qrc_u32* map, float* amax, float* scale, qrc_u32 mode) {
    qrc::reduce_run<qrc::OpAbsBF16>(in, n, map, amax, scale, mode);
}

__global__ void qrc_k_set_word(qrc_u32* map, qrc_u32 idx, qrc_u32 val) { map[idx] = val; }

// e4m3x2 pack: upper byte from `hi`, lower byte from `lo`; RNE, saturating.
static __device__ __forceinline__ unsigned short cvt_e4m3x2(float hi, float lo) {
    unsigned short r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

// Two bf16 (one 32-bit word, element 0 in the low half) -> two e4m3 bytes.
static __device__ __forceinline__ unsigned short quant_word(qrc_u32 w, float s) {
    const float f0 = __uint_as_float(w << 16), f1 = __uint_as_float(w & 0xFFFF0000u);
    return cvt_e4m3x2(__fmul_rn(f1, s), __fmul_rn(f0, s));
}

// Quantize pass: 8 bf16 (16 B) in -> 8 e4m3 (8 B) out per unit, four units in
// flight per thread.  Units are walked from the top of the buffer down: the
// amax pass just before ended at the top, so the first ~100 MB this pass reads
// are still in the 126 MB L2.  Output stores are streaming (evict-first).
// Vector path needs in % 16 == 0 and q % 8 == 0; any other alignment takes the
// element path.
__global__ void __launch_bounds__(512, 2)
qrc_k_quant_e4m3(const uint16_t* in, qrc_u64 n, uint8_t* q, const float* scale_p) {
    qrc::griddep_wait();                     // the scale comes from the amax launch before
    const float s = *scale_p;
    const qrc_u64 tid = (qrc_u64)blockIdx.x * blockDim.x + threadIdx.x;
    const qrc_u64 stride = (qrc_u64)gridDim.x * blockDim.x;
    const bool vec = (((qrc_u64)in & 15) == 0) && (((qrc_u64)q & 7) == 0);
    const qrc_u64 nv = vec ? n / 8 : 0;
    for (qrc_u64 i = tid; i < nv; i += 4 * stride) {
        uint4 v[4];
        #pragma unroll
        for (int u = 0; u < 4; u++) {
            const qrc_u64 j = i + u * stride;
            if (j < nv) v[u] = qrc::ld_stream16((qrc_u64)(in + 8 * (nv - 1 - j)));
        }
        #pragma unroll
        for (int u = 0; u < 4; u++) {
            const qrc_u64 j = i + u * stride;
            if (j < nv) {
                uint2 o;
                o.x = (qrc_u32)quant_word(v[u].x, s) | ((qrc_u32)quant_word(v[u].y, s) << 16);
                o.y = (qrc_u32)quant_word(v[u].z, s) | ((qrc_u32)quant_word(v[u].w, s) << 16);
                __stcs((uint2*)(q + 8 * (nv - 1 - j)), o);
            }
        }
    }
    for (qrc_u64 e = nv * 8 + tid; e < n; e += stride) {
        const float f = __uint_as_float((qrc_u32)in[e] << 16);
        q[e] = (uint8_t)(cvt_e4m3x2(0.0f, __fmul_rn(f, s)) & 0xFFu);
    }
}

// Side-aware quantize pass (the input has a side map).  Each 256-thread group
// claims 64 KiB input blocks (8 pairs of 4 KiB chunks) from its side's queue,
// top-down (the end of the input is the part the amax pass left in L2), and
// converts the 4 KiB chunk of every pair that is homed on its own die: reads
// stay on the die, only the half-size e4m3 stores may cross.  A group whose
// queue is empty helps the other side.  The last CTA (ticket) resets the
// queues for the next launch.  Needs in % 16 == 0, q % 8 == 0, 4 KiB chunks
// and 1024-thread blocks; the host uses qrc_k_quant_e4m3 otherwise.
static __device__ __forceinline__ void quant16(const uint4 v, float s, uint8_t* dst) {
    uint2 o;
    o.x = (qrc_u32)quant_word(v.x, s) | ((qrc_u32)quant_word(v.y, s) << 16);
    o.y = (qrc_u32)quant_word(v.z, s) | ((qrc_u32)quant_word(v.w, s) << 16);
    __stcs((uint2*)dst, o);
}

__global__ void __launch_bounds__(1024, 1)
qrc_k_quant_e4m3_sa(const uint16_t* in, qrc_u64 n, uint8_t* q, const float* scale_p, qrc_u32* map, qrc_u32 mode) {
    using namespace qrc;
    const qrc_u64 a = (qrc_u64)in, end = a + 2 * n;
    ChunkMap cm;
    cm.setup(a, end, map, mode & ~SCHED_MASK);      // header only: written by discovery alone
    griddep_wait();                                 // the scale, and the queues' reset
    const float s = *scale_p;
    __shared__ qrc_u32 s_claim[2][4];
    const int g = threadIdx.x >> 8, t = threadIdx.x & 255;
    const bool leader = t == 0;
    const qrc_u64 nb = (cm.npairs + 7) >> 3;
    const bool fast = (cm.lo & 0xFFFFull) == 0;
    qrc_u32 pat = 0;
    #pragma unroll
    for (int j = 0; j < 8; j++) pat |= (qrc_u32)parity64(((qrc_u64)j << 13) & cm.mask) << j;
    int side = cm.side;
    qrc_u32* queue = &map[side ? H_QUEUE1 : H_QUEUE0];
    bool stealing = false;
    int par = 0;
    if (leader) s_claim[0][g] = atomicAdd(queue, 1u);
    group_bar(g);
    qrc_u32 cur = s_claim[0][g];
    for (;;) {
        qrc_u32 nxt = 0;
        if (cur >= nb) {
            if (stealing) break;
            stealing = true;
            side ^= 1;
            queue = &map[side ? H_QUEUE1 : H_QUEUE0];
            if (leader) nxt = atomicAdd(queue, 1u);
        } else {
            if (leader) nxt = atomicAdd(queue, 1u);
            const qrc_u64 p0 = (nb - 1 - cur) << 3;            // top-down
            uint4 v[8];
            qrc_u64 x[8];
            if (fast && p0 + 8 <= cm.npairs) {
                const qrc_u64 base = cm.lo + (p0 << 13);
                int pbit = 0;
                if (cm.use_page_bits) {
                    const qrc_u64 pg = (base - cm.page_base) >> 21;
                    pbit = (int)(cm.page_bits[pg >> 5] >> (pg & 31)) & 1;
                }
                const qrc_u32 second = (qrc_u32)(parity64(base & cm.mask) ^ pbit ^ cm.flip ^ side) ? ~pat : pat;
                #pragma unroll
                for (int j = 0; j < 8; j++) {
                    x[j] = base + 16ull * t + ((qrc_u64)j << 13) + ((qrc_u64)((second >> j) & 1u) << 12);
                    v[j] = ld_stream16(x[j]);
                }
            } else {
                #pragma unroll
                for (int j = 0; j < 8; j++) {
                    x[j] = 0;
                    if (p0 + j < cm.npairs) {
                        x[j] = cm.chunk_of(p0 + j, side) + 16ull * t;
                        v[j] = ld_stream16(x[j]);
                    }
                }
            }
            #pragma unroll
            for (int j = 0; j < 8; j++)
                if (x[j]) quant16(v[j], s, q + ((x[j] - a) >> 1));
        }
        par ^= 1;
        if (leader) s_claim[par][g] = nxt;
        group_bar(g);
        cur = s_claim[par][g];
    }
    // Elements outside the whole pairs: CTA 0 takes the head, the last CTA the tail.
    if (blockIdx.x == 0) {
        for (qrc_u64 e = threadIdx.x; e < (cm.lo - a) >> 1; e += blockDim.x)
            q[e] = (uint8_t)(cvt_e4m3x2(0.0f, __fmul_rn(__uint_as_float((qrc_u32)in[e] << 16), s)) & 0xFFu);
    }
    if (blockIdx.x == gridDim.x - 1) {
        for (qrc_u64 e = ((cm.hi - a) >> 1) + threadIdx.x; e < n; e += blockDim.x)
            q[e] = (uint8_t)(cvt_e4m3x2(0.0f, __fmul_rn(__uint_as_float((qrc_u32)in[e] << 16), s)) & 0xFFu);
    }
    griddep_launch_dependents();
    __syncthreads();
    if (threadIdx.x == 0) {
        qrc_u32 tk;
        asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;"
                     : "=r"(tk) : "l"(&map[H_QUANT_TICKET]), "r"(gridDim.x - 1) : "memory");
        if (tk == gridDim.x - 1) {                      // every claim is done: reset for the next launch
            map[H_QUEUE0] = 0u;
            map[H_QUEUE1] = 0u;
        }
    }
}

// ---- single-launch fused amax -> e4m3 --------------------------------------
//
// One launch of one 1024-thread CTA per SM, four 256-thread groups per CTA;
// every group reads the 4 KiB chunk of its die in each of the 8 pairs of a
// 64 KiB block (128 B per thread), like the reduction's walk.
//   Phase 1 (amax).  The first 3 * 4 * K_s blocks of side s are shared out
//     statically: the CTA on SM (s, k) reads blocks k*4 + g + i*4*K_s for
//     i < kFusedStash with its group g and keeps them on the chip, the first
//     two in tensor memory (tcgen05.st into the thread's TMEM lane, 64
//     columns per warp, all 512 columns per CTA) and the third in shared
//     memory (128 KiB per CTA).  The rest of the blocks are claimed one per
//     group from the side's queue in increasing order (a side whose queue is
//     empty helps the other), so slower SMs are absorbed; the last 4 * K_s
//     blocks of a side go out as halves (fused_unit).  The top
//     QRC_FUSED_L2_MB of the input is read with the default L2 policy and
//     everything else evict-first, so L2 keeps what was read last.
//   Grid barrier (bounded).  Every CTA adds its block maximum to the map and
//     arrives; all wait until every CTA has arrived.  Each group's first
//     phase-2 block (claimed during phase 1; claims and loads need no amax)
//     is already loading while it waits.
//   Phase 2 (quantize).  The claimed blocks again, from a second pair of
//     queues, top-down: the blocks read last in phase 1, those still in L2,
//     come first.  Group g quantizes its stash block i after g + 2i claimed
//     blocks, so at any moment most warps have HBM loads in flight.
// About 58 MB of a 268 MB input never cross HBM twice.  Edges outside the
// 64 KiB-aligned body are handled by CTA 0 element by element in both
// phases.  The last CTA to finish (ticket) publishes amax and scale and
// resets the map words for the next launch.  If the barrier wait gives up
// (about 1 s) or a static share was not read, amax is NaN (scale 1, as in the
// two-launch path), the quantize is skipped and the sticky word H_WAIT_ERR
// gets bit 1; tensor memory is freed on every path.
constexpr int kFusedTmemIters = 2;
constexpr int kFusedSmemIters = 1;
constexpr int kFusedStash = kFusedTmemIters + kFusedSmemIters;
constexpr qrc_u32 kFusedSmemBytes = 1024u * 128u * kFusedSmemIters;
constexpr long long kFusedWaitCycles = 1ll << 31;          // about one second
#ifndef QRC_FUSED_L2_MB
#define QRC_FUSED_L2_MB 96
#endif
constexpr qrc_u64 kFusedL2Blocks = (qrc_u64)QRC_FUSED_L2_MB << 4;   // 64 KiB blocks
// Phase 2: group g quantizes stash block i after QRC_FUSED_STASH_G * g +
// QRC_FUSED_STASH_I * i of its claimed blocks.
#ifndef QRC_FUSED_STASH_G
#define QRC_FUSED_STASH_G 1
#endif
#ifndef QRC_FUSED_STASH_I
#define QRC_FUSED_STASH_I 2
#endif

static __device__ __forceinline__ void tmem_st_x32(qrc_u32 taddr, const uint4 (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
                 "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
                 "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n\t"
                 "tcgen05.wait::st.sync.aligned;"
                 :: "r"(taddr),
                    "r"(v[0].x), "r"(v[0].y), "r"(v[0].z), "r"(v[0].w), "r"(v[1].x), "r"(v[1].y), "r"(v[1].z), "r"(v[1].w),
                    "r"(v[2].x), "r"(v[2].y), "r"(v[2].z), "r"(v[2].w), "r"(v[3].x), "r"(v[3].y), "r"(v[3].z), "r"(v[3].w),
                    "r"(v[4].x), "r"(v[4].y), "r"(v[4].z), "r"(v[4].w), "r"(v[5].x), "r"(v[5].y), "r"(v[5].z), "r"(v[5].w),
                    "r"(v[6].x), "r"(v[6].y), "r"(v[6].z), "r"(v[6].w), "r"(v[7].x), "r"(v[7].y), "r"(v[7].z), "r"(v[7].w)
                 : "memory");
}
static __device__ __forceinline__ void tmem_ld_x8(qrc_u32 taddr, uint4 (&v)[2]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
                 "tcgen05.wait::ld.sync.aligned;"
                 : "=r"(v[0].x), "=r"(v[0].y), "=r"(v[0].z), "=r"(v[0].w), "=r"(v[1].x), "=r"(v[1].y), "=r"(v[1].z), "=r"(v[1].w)
                 : "r"(taddr) : "memory");
}

// Which half of each of the 8 pairs of the 64 KiB block at `base` is homed
// on side s: bit j set means the second 4 KiB chunk of pair j.
static __device__ __forceinline__ qrc_u32 fused_second(const qrc::ChunkMap& cm, qrc_u64 base, int s, qrc_u32 pat) {
    int pbit = 0;
    if (cm.use_page_bits) {
        const qrc_u64 pg = (base - cm.page_base) >> 21;
        pbit = (int)(cm.page_bits[pg >> 5] >> (pg & 31)) & 1;
    }
    return (qrc_u32)(qrc::parity64(base & cm.mask) ^ pbit ^ cm.flip ^ s) ? ~pat : pat;
}
static __device__ __forceinline__ qrc_u64 fused_addr(qrc_u64 row, qrc_u32 second, int j) {
    return row + ((qrc_u64)j << 13) + ((qrc_u64)((second >> j) & 1u) << 12);
}
// Claim units of a side's queue in the fused kernel (blocks [dyn, nbf) of a
// side with K SMs, nd of them): the first nd - T are whole 64 KiB blocks, then
// 2T halves (4 pairs each) of the last T = min(4K, nd) blocks in claim order, so the end of each phase balances to half a block.  Sets the
// block's position in claim order and the half (-1 for a whole block);
// false when the queue is exhausted.
static __device__ __forceinline__ bool fused_unit(qrc_u32 cur, qrc_u32 nbf, qrc_u32 dyn, qrc_u32 K, qrc_u32& pos,
                                                  int& half) {
    const qrc_u32 nd = nbf - dyn, T = 4u * K < nd ? 4u * K : nd, F = nd - T;
    if (cur < F) { pos = cur; half = -1; return true; }
    const qrc_u32 h = cur - F;
    if (h >= 2u * T) return false;
    pos = F + (h >> 1);
    half = (int)(h & 1u);
    return true;
}

static __device__ __forceinline__ uint8_t quant_one(uint16_t x, float s) {
    return (uint8_t)(cvt_e4m3x2(0.0f, __fmul_rn(__uint_as_float((qrc_u32)x << 16), s)) & 0xFFu);
}

__global__ void __launch_bounds__(1024, 1)
qrc_k_amax_quant_fused(const uint16_t* in, qrc_u64 n, uint8_t* q, float* amax_out, float* scale_out, qrc_u32* map,
                       qrc_u32 mode) {
    using namespace qrc;
    extern __shared__ __align__(128) uint4 s_stash[];          // kFusedSmemIters x 8 x 1024 uint4
    __shared__ qrc_u32 s_taddr;
    __shared__ qrc_u32 s_claim[2][4];
    __shared__ qrc_u32 s_first2[4];                            // each group's first phase-2 claim
    __shared__ float s_scale;
    __shared__ int s_ok, s_last;
    const int tid = threadIdx.x, warp = tid >> 5, g = tid >> 8, t = tid & 255;
    const bool leader = t == 0;
    const qrc_u64 a = (qrc_u64)in, end = a + 2 * n;
    ChunkMap cm;
    cm.setup(a, end, map, mode & ~SCHED_MASK);                 // header only: written by discovery alone
    const qrc_u32 k0 = map[H_NSIDE0], k1 = map[H_NSIDE1];
    const int own_side = cm.side, k = cm.sm_index;
    const qrc_u32 Ks = own_side ? k1 : k0;
    const bool has_share = cm.aware && k >= 0 && (qrc_u32)k < Ks && k0 <= 128u && k1 <= 128u;
    const qrc_u64 lo64 = (a + 0xFFFFull) & ~0xFFFFull;
    // Block indices are 32-bit: the host sends inputs of at most 2^47 bytes here.
    const qrc_u32 nbf = end > lo64 ? (qrc_u32)((end - lo64) >> 16) : 0u;   // whole 64 KiB blocks of the body
    const qrc_u64 body_end = lo64 + ((qrc_u64)nbf << 16);
    // blocks [0, dyn_s) of side s are the static stash shares, [dyn_s, nbf) are claimed
    const qrc_u32 dyn0 = kFusedStash * 4u * k0 < nbf ? kFusedStash * 4u * k0 : nbf;
    const qrc_u32 dyn1 = kFusedStash * 4u * k1 < nbf ? kFusedStash * 4u * k1 : nbf;
    const qrc_u32 own_dyn = own_side ? dyn1 : dyn0;
    const qrc_u32 l2_from = nbf > (qrc_u32)kFusedL2Blocks ? nbf - (qrc_u32)kFusedL2Blocks : 0u;

    qrc_u32 pat = 0;
    #pragma unroll
    for (int j = 0; j < 8; j++) pat |= (qrc_u32)parity64(((qrc_u64)j << 13) & cm.mask) << j;

    // Tensor memory: all 512 columns; warp w owns lanes (w % 4) * 32 .. + 31
    // of columns (w / 4) * 64 .. + 63, i.e. two 32-column slots per thread.
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;"
                     :: "r"((qrc_u32)__cvta_generic_to_shared(&s_taddr)) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const qrc_u32 tslot = s_taddr + ((qrc_u32)((warp & 3) * 32) << 16) + (qrc_u32)(warp >> 2) * 64u;
    griddep_wait();
#if QRC_TIMELINE
    // Diagnostic build: per CTA, %globaltimer (ns, low 32 bits) at the start
    // of phase 1, the arrival at the barrier, its release and the end of
    // phase 2, in map words O_TIMELINE + 4 * CTA.
    qrc_u32 tl0;
    asm volatile("{\n\t.reg .u64 t;\n\tmov.u64 t, %%globaltimer;\n\tcvt.u32.u64 %0, t;\n\t}" : "=r"(tl0));
#endif

    // ---- phase 1: amax ---------------------------------------------------------
    qrc_u32 acc = 0;                                           // two bf16 lanes of max |x|
    for (int i = 0; i < kFusedStash; i++) {                    // the static shares, kept on the chip
        const qrc_u32 b = (qrc_u32)k * 4u + (qrc_u32)g + (qrc_u32)i * 4u * Ks;
        if (!has_share || b >= own_dyn) break;                 // the same for the whole group
        const qrc_u64 base = lo64 + ((qrc_u64)b << 16);
        const qrc_u32 second = fused_second(cm, base, own_side, pat);
        const qrc_u64 row = base + 16ull * t;
        uint4 v[8];
        #pragma unroll
        for (int j = 0; j < 8; j++) v[j] = ld16<2>(fused_addr(row, second, j));
        #pragma unroll
        for (int j = 0; j < 8; j++) acc = OpAbsBF16::step16(acc, v[j]);
        if (i < kFusedTmemIters) {
            tmem_st_x32(tslot + 32u * (qrc_u32)i, v);
        } else {
            uint4* sp = s_stash + (size_t)(i - kFusedTmemIters) * 8192 + tid;
            #pragma unroll
            for (int j = 0; j < 8; j++) sp[j * 1024] = v[j];
        }
    }
    // The group's first phase-2 claim goes out now (it needs no amax); its
    // reply is read after the group barriers of the loop below.
    if (leader) s_first2[g] = atomicAdd(&map[own_side ? H_FUSED_Q1 : H_FUSED_Q0], 1u);
    int par = 0;                                               // s_claim slot of the group's last read
    {                                                          // the claimed blocks, bottom-up
        int side = own_side;
        bool stealing = false;
        qrc_u32* queue = &map[side ? H_QUEUE1 : H_QUEUE0];
        if (leader) s_claim[0][g] = atomicAdd(queue, 1u);
        group_bar(g);
        qrc_u32 cur = s_claim[0][g];
        for (;;) {
            const qrc_u32 dyn = side ? dyn1 : dyn0;
            qrc_u32 nxt = 0, pos;
            int half;
            if (!fused_unit(cur, nbf, side ? dyn1 : dyn0, side ? k1 : k0, pos, half)) {
                if (stealing) break;
                stealing = true;
                side ^= 1;
                queue = &map[side ? H_QUEUE1 : H_QUEUE0];
                if (leader) nxt = atomicAdd(queue, 1u);
            } else {
                if (leader) nxt = atomicAdd(queue, 1u);
                const qrc_u32 b = dyn + pos;
                const qrc_u64 base = lo64 + ((qrc_u64)b << 16);
                // a half block is pairs 4*half .. 4*half+3: shift the pattern and the row
                const int j0 = half < 0 ? 0 : 4 * half, jn = half < 0 ? 8 : 4;
                const qrc_u32 second = fused_second(cm, base, side, pat) >> j0;
                const qrc_u64 row = base + 16ull * t + ((qrc_u64)j0 << 13);
                uint4 v[8];
                if (b >= l2_from) {
                    #pragma unroll
                    for (int j = 0; j < 8; j++) v[j] = j < jn ? ld16<1>(fused_addr(row, second, j)) : make_uint4(0, 0, 0, 0);
                } else {
                    #pragma unroll
                    for (int j = 0; j < 8; j++) v[j] = j < jn ? ld16<2>(fused_addr(row, second, j)) : make_uint4(0, 0, 0, 0);
                }
                #pragma unroll
                for (int j = 0; j < 8; j++) acc = OpAbsBF16::step16(acc, v[j]);
            }
            par ^= 1;                                          // a slot is rewritten two barriers after it was read
            if (leader) s_claim[par][g] = nxt;
            group_bar(g);
            cur = s_claim[par][g];
        }
    }
    // Phase 2's first block is loaded now, so its loads are in flight across
    // the barrier; the second claim goes out too.  The claim goes into the
    // slot the group read two barriers ago (a lagging thread may still read
    // the other one).
    par ^= 1;
    if (leader) s_claim[par][g] = atomicAdd(&map[own_side ? H_FUSED_Q1 : H_FUSED_Q0], 1u);
    uint4 pv[8];
    qrc_u32 pos1;
    int half1;
    const bool have1 = fused_unit(s_first2[g], nbf, own_dyn, Ks, pos1, half1);
    const int pj0 = half1 < 0 ? 0 : 4 * half1, pjn = have1 ? (half1 < 0 ? 8 : 4) : 0;
    qrc_u64 prow = 0;
    qrc_u32 psecond = 0;
    if (have1) {
        const qrc_u64 base = lo64 + ((qrc_u64)(nbf - 1 - pos1) << 16);   // top-down
        psecond = fused_second(cm, base, own_side, pat) >> pj0;
        prow = base + 16ull * t + ((qrc_u64)pj0 << 13);
        #pragma unroll
        for (int j = 0; j < 8; j++) if (j < pjn) pv[j] = ld16<2>(fused_addr(prow, psecond, j));
    }
    // Edges, element by element: [a, lo64) and [body_end, end), both empty or
    // shorter than 64 KiB (when end <= lo64 the head is the whole input).
    const qrc_u64 head_n = ((lo64 < end ? lo64 : end) - a) >> 1, tail_e = (body_end - a) >> 1;
    if (blockIdx.x == 0) {
        for (qrc_u64 e = tid; e < head_n; e += blockDim.x) acc = absmax_step_bf16x2(acc, (qrc_u32)in[e]);
        for (qrc_u64 e = tail_e + tid; e < n; e += blockDim.x) acc = absmax_step_bf16x2(acc, (qrc_u32)in[e]);
    }

    // ---- grid barrier ------------------------------------------------------------
    // Every CTA adds its maximum and its share bit, then arrives; all wait
    // (bounded) until every CTA has arrived.
    const qrc_u32 v = block_max(OpAbsBF16::to_red(acc));
#if QRC_TIMELINE
    qrc_u32 tl1, tl2, tl3;
    asm volatile("{\n\t.reg .u64 t;\n\tmov.u64 t, %%globaltimer;\n\tcvt.u32.u64 %0, t;\n\t}" : "=r"(tl1));
#endif
    if (tid == 0) {
        asm volatile("red.relaxed.gpu.global.max.u32 [%0], %1;" :: "l"(&map[H_FUSED_ACC]), "r"(v) : "memory");
        if (has_share) atomicOr(&map[O_FUSED_SHARES + ((qrc_u32)own_side * 128u + (qrc_u32)k) / 32u], 1u << (k & 31));
        qrc_u32 arrived;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(arrived) : "l"(&map[H_FUSED_ARRIVE]) : "memory");
        bool ok = true;
        if (arrived != gridDim.x - 1) {
            const long long t0 = clock64();
            for (;;) {
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(arrived) : "l"(&map[H_FUSED_ARRIVE]) : "memory");
                if (arrived >= gridDim.x) break;
                if (clock64() - t0 > kFusedWaitCycles) { ok = false; break; }
            }
        }
        float amax = __int_as_float(0x7FFFFFFF);
        if (ok) {
            amax = __uint_as_float(__ldcg(&map[H_FUSED_ACC]));
            for (int w = 0; w < 8; w++) {                       // every static share of both sides was read
                const qrc_u32 K = (w >> 2) ? k1 : k0, lo = (qrc_u32)(w & 3) * 32u;
                const qrc_u32 req = K <= lo ? 0u : (K - lo >= 32u ? 0xFFFFFFFFu : (1u << (K - lo)) - 1u);
                if ((__ldcg(&map[O_FUSED_SHARES + w]) & req) != req) ok = false;
            }
        }
        if (!ok) atomicExch(&map[H_FUSED_ERR], 1u);
        s_ok = ok;
        s_scale = e4m3_scale_from_amax(amax);
    }
    __syncthreads();
#if QRC_TIMELINE
    asm volatile("{\n\t.reg .u64 t;\n\tmov.u64 t, %%globaltimer;\n\tcvt.u32.u64 %0, t;\n\t}" : "=r"(tl2));
#endif

    // ---- phase 2: quantize the claimed blocks top-down, and the stash --------
    // Group g quantizes its stash block i between its claimed blocks, after
    // g + 2i of them, so at any moment most warps of an SM have HBM loads in
    // flight while the others work from the chip; what is left of the stash
    // (a group with fewer claims) follows the claims.
    if (s_ok) {
        const float sc = s_scale;
        int ns = 0;                                            // stash blocks of this group
        #pragma unroll
        for (int i = 0; i < kFusedStash; i++)
            ns += (has_share && (qrc_u32)k * 4u + (qrc_u32)g + (qrc_u32)i * 4u * Ks < own_dyn) ? 1 : 0;
        auto stash_block = [&](int i) {                        // quantize stash block i, a quarter at a time
            const qrc_u32 b = (qrc_u32)k * 4u + (qrc_u32)g + (qrc_u32)i * 4u * Ks;
            const qrc_u64 base = lo64 + ((qrc_u64)b << 16);
            const qrc_u32 second = fused_second(cm, base, own_side, pat);
            const qrc_u64 row = base + 16ull * t;
            #pragma unroll 1
            for (int h = 0; h < 4; h++) {
                uint4 w[2];
                if (i < kFusedTmemIters) {
                    tmem_ld_x8(tslot + 32u * (qrc_u32)i + 8u * (qrc_u32)h, w);
                } else {
                    const uint4* sp = s_stash + (size_t)(i - kFusedTmemIters) * 8192 + (size_t)h * 2048 + tid;
                    w[0] = sp[0];
                    w[1] = sp[1024];
                }
                quant16(w[0], sc, q + ((fused_addr(row, second, 2 * h) - a) >> 1));
                quant16(w[1], sc, q + ((fused_addr(row, second, 2 * h + 1) - a) >> 1));
            }
        };
        int si = 0, done = 0;
        if (have1) {                                           // the block loaded before the barrier
            if (si < ns && done == QRC_FUSED_STASH_G * g + QRC_FUSED_STASH_I * si) stash_block(si++);
            #pragma unroll
            for (int j = 0; j < 8; j++)
                if (j < pjn) quant16(pv[j], sc, q + ((fused_addr(prow, psecond, j) - a) >> 1));
            done++;
        }
        int side = own_side;
        bool stealing = false;
        qrc_u32* queue = &map[side ? H_FUSED_Q1 : H_FUSED_Q0];
        qrc_u32 cur = s_claim[par][g];                         // the second claim, made before the barrier
        for (;;) {
            qrc_u32 nxt = 0, pos;
            int half;
            if (!fused_unit(cur, nbf, side ? dyn1 : dyn0, side ? k1 : k0, pos, half)) {
                if (stealing) break;
                stealing = true;
                side ^= 1;
                queue = &map[side ? H_FUSED_Q1 : H_FUSED_Q0];
                if (leader) nxt = atomicAdd(queue, 1u);
            } else {
                if (leader) nxt = atomicAdd(queue, 1u);
                const qrc_u32 b = nbf - 1 - pos;              // top-down
                const qrc_u64 base = lo64 + ((qrc_u64)b << 16);
                const int j0 = half < 0 ? 0 : 4 * half, jn = half < 0 ? 8 : 4;
                const qrc_u32 second = fused_second(cm, base, side, pat) >> j0;
                const qrc_u64 row = base + 16ull * t + ((qrc_u64)j0 << 13);
                if (si < ns && done == QRC_FUSED_STASH_G * g + QRC_FUSED_STASH_I * si) stash_block(si++);
                uint4 v[8];
                #pragma unroll
                for (int j = 0; j < 8; j++) if (j < jn) v[j] = ld16<2>(fused_addr(row, second, j));
                #pragma unroll
                for (int j = 0; j < 8; j++)
                    if (j < jn) quant16(v[j], sc, q + ((fused_addr(row, second, j) - a) >> 1));
                done++;
            }
            par ^= 1;
            if (leader) s_claim[par][g] = nxt;
            group_bar(g);
            cur = s_claim[par][g];
        }
        while (si < ns) stash_block(si++);
#if QRC_TIMELINE
        // Diagnostic build: per group, the end of its phase-2 work, its claims
        // and how many of them came from the other side's queue, in map words
        // O_PAGE_LAT + 2 * (4 * CTA + group) (discovery's diagnostics area).
        if (leader && blockIdx.x < 148) {
            qrc_u32 tg;
            asm volatile("{\n\t.reg .u64 t;\n\tmov.u64 t, %%globaltimer;\n\tcvt.u32.u64 %0, t;\n\t}" : "=r"(tg));
            map[O_PAGE_LAT + 2 * (4 * blockIdx.x + g)] = tg;
            map[O_PAGE_LAT + 2 * (4 * blockIdx.x + g) + 1] = (qrc_u32)done | ((qrc_u32)stealing << 16);
        }
#endif
        if (blockIdx.x == 0) {
            for (qrc_u64 e = tid; e < head_n; e += blockDim.x) q[e] = quant_one(in[e], sc);
            for (qrc_u64 e = tail_e + tid; e < n; e += blockDim.x) q[e] = quant_one(in[e], sc);
        }
    }

    // ---- tensor memory back, then the last CTA publishes and resets -------------
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
#if QRC_TIMELINE
    asm volatile("{\n\t.reg .u64 t;\n\tmov.u64 t, %%globaltimer;\n\tcvt.u32.u64 %0, t;\n\t}" : "=r"(tl3));
    if (tid == 0 && blockIdx.x < 256) {
        qrc_u32* tl = map + O_TIMELINE + 4 * blockIdx.x;
        tl[0] = tl0; tl[1] = tl1; tl[2] = tl2; tl[3] = tl3;
    }
#endif
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" :: "r"(s_taddr) : "memory");
    }
    griddep_launch_dependents();
    if (tid == 0) {
        qrc_u32 tk;
        asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;"
                     : "=r"(tk) : "l"(&map[H_FUSED_DONE]), "r"(gridDim.x - 1) : "memory");
        s_last = tk == gridDim.x - 1;
    }
    __syncthreads();
    if (s_last && tid == 0) {
        const bool err = __ldcg(&map[H_FUSED_ERR]) != 0u;
        const float amax = err ? __int_as_float(0x7FFFFFFF) : __uint_as_float(__ldcg(&map[H_FUSED_ACC]));
        *amax_out = amax;
        *scale_out = e4m3_scale_from_amax(amax);              // 1 for a NaN amax, as in the two-launch path
        if (err) map[H_WAIT_ERR] |= 2u;                        // sticky record for diagnostics
        map[H_FUSED_ERR] = 0u;
        map[H_FUSED_ACC] = 0u;
        map[H_FUSED_ARRIVE] = 0u;
        map[H_QUEUE0] = 0u;
        map[H_QUEUE1] = 0u;
        map[H_FUSED_Q0] = 0u;
        map[H_FUSED_Q1] = 0u;
        for (int w = 0; w < 8; w++) map[O_FUSED_SHARES + w] = 0u;
    }
}

// Side-aware copy y = x: the same group claims as qrc_k_quant_e4m3_sa, each
// group copying the 4 KiB chunk of every pair that is homed on its die.  With
// y from qrc_alloc_like (same offset in its 2 MiB page, pages homed like
// x's), the stores stay on the die as well.
__global__ void __launch_bounds__(1024, 1)
qrc_k_copy_f32_sa(const float* x, qrc_u64 n, float* y, qrc_u32* map, qrc_u32 mode) {
    using namespace qrc;
    const qrc_u64 a = (qrc_u64)x, end = a + 4 * n, yo = (qrc_u64)y - a;
    ChunkMap cm;
    cm.setup(a, end, map, mode & ~SCHED_MASK);
    griddep_wait();
    __shared__ qrc_u32 s_claim[2][4];
    const int g = threadIdx.x >> 8, t = threadIdx.x & 255;
    const bool leader = t == 0;
    const qrc_u64 nb = (cm.npairs + 7) >> 3;
    const bool fast = (cm.lo & 0xFFFFull) == 0;
    qrc_u32 pat = 0;
    #pragma unroll
    for (int j = 0; j < 8; j++) pat |= (qrc_u32)parity64(((qrc_u64)j << 13) & cm.mask) << j;
    int side = cm.side;
    qrc_u32* queue = &map[side ? H_QUEUE1 : H_QUEUE0];
    bool stealing = false;
    int par = 0;
    if (leader) s_claim[0][g] = atomicAdd(queue, 1u);
    group_bar(g);
    qrc_u32 cur = s_claim[0][g];
    for (;;) {
        qrc_u32 nxt = 0;
        if (cur >= nb) {
            if (stealing) break;
            stealing = true;
            side ^= 1;
            queue = &map[side ? H_QUEUE1 : H_QUEUE0];
            if (leader) nxt = atomicAdd(queue, 1u);
        } else {
            if (leader) nxt = atomicAdd(queue, 1u);
            const qrc_u64 p0 = (qrc_u64)cur << 3;
            uint4 v[8];
            qrc_u64 xa[8];
            if (fast && p0 + 8 <= cm.npairs) {
                const qrc_u64 base = cm.lo + (p0 << 13);
                int pbit = 0;
                if (cm.use_page_bits) {
                    const qrc_u64 pg = (base - cm.page_base) >> 21;
                    pbit = (int)(cm.page_bits[pg >> 5] >> (pg & 31)) & 1;
                }
                const qrc_u32 second = (qrc_u32)(parity64(base & cm.mask) ^ pbit ^ cm.flip ^ side) ? ~pat : pat;
                #pragma unroll
                for (int j = 0; j < 8; j++) {
                    xa[j] = base + 16ull * t + ((qrc_u64)j << 13) + ((qrc_u64)((second >> j) & 1u) << 12);
                    v[j] = ld_stream16(xa[j]);
                }
            } else {
                #pragma unroll
                for (int j = 0; j < 8; j++) {
                    xa[j] = 0;
                    if (p0 + j < cm.npairs) {
                        xa[j] = cm.chunk_of(p0 + j, side) + 16ull * t;
                        v[j] = ld_stream16(xa[j]);
                    }
                }
            }
            #pragma unroll
            for (int j = 0; j < 8; j++)
                if (xa[j]) __stcs((uint4*)(xa[j] + yo), v[j]);
        }
        par ^= 1;
        if (leader) s_claim[par][g] = nxt;
        group_bar(g);
        cur = s_claim[par][g];
    }
    if (blockIdx.x == 0)
        for (qrc_u64 e = threadIdx.x; e < (cm.lo - a) >> 2; e += blockDim.x) y[e] = x[e];
    if (blockIdx.x == gridDim.x - 1)
        for (qrc_u64 e = ((cm.hi - a) >> 2) + threadIdx.x; e < n; e += blockDim.x) y[e] = x[e];
    griddep_launch_dependents();
    __syncthreads();
    if (threadIdx.x == 0) {
        qrc_u32 tk;
        asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;"
                     : "=r"(tk) : "l"(&map[H_COPY_TICKET]), "r"(gridDim.x - 1) : "memory");
        if (tk == gridDim.x - 1) {
            map[H_QUEUE0] = 0u;
            map[H_QUEUE1] = 0u;
        }
    }
}

// Plain streaming read of [p, p + bytes) with no side logic: a grid-stride
// walk over 16-byte units, D loads in flight per thread, folded by XOR into
// one word per warp (so the loads cannot be dropped).  A measuring stick for
// what a read-only stream reaches on this GPU; the tail (bytes % 16) is left
// out.
template <int D, int T, int B>
__global__ void __launch_bounds__(T, B)
qrc_k_read_stream(const uint4* p, qrc_u64 nv, qrc_u32* sink) {
    const qrc_u64 tid = (qrc_u64)blockIdx.x * blockDim.x + threadIdx.x;
    const qrc_u64 stride = (qrc_u64)gridDim.x * blockDim.x;
    qrc_u32 x = 0;
    for (qrc_u64 i = tid; i < nv; i += D * stride) {
        uint4 v[D];
        #pragma unroll
        for (int u = 0; u < D; u++) {
            const qrc_u64 j = i + u * stride;
            v[u] = j < nv ? qrc::ld_stream16((qrc_u64)(p + j)) : make_uint4(0, 0, 0, 0);
        }
        #pragma unroll
        for (int u = 0; u < D; u++) x ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
    }
    x = __reduce_xor_sync(0xFFFFFFFFu, x);
    if ((threadIdx.x & 31) == 0) atomicXor(sink, x);
}

__global__ void qrc_k_debug_cvt_e4m3(const float* in, qrc_u64 n, uint8_t* out) {
    for (qrc_u64 i = (qrc_u64)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (qrc_u64)gridDim.x * blockDim.x)
        out[i] = (uint8_t)(cvt_e4m3x2(0.0f, in[i]) & 0xFFu);
}

__global__ void qrc_k_fill_uniform(float* out, qrc_u64 n, qrc_u64 key, qrc_u64 offset) {
    for (qrc_u64 i = (qrc_u64)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (qrc_u64)gridDim.x * blockDim.x)
        out[i] = qrc_gen::uniform_pm1(key, offset + i);
}
__global__ void qrc_k_fill_normal(float* out, qrc_u64 n, qrc_u64 key, qrc_u64 offset, float sigma) {
    for (qrc_u64 i = (qrc_u64)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (qrc_u64)gridDim.x * blockDim.x)
        out[i] = qrc_gen::normal01(key, offset + i) * sigma;
}
__global__ void qrc_k_fill_normal_bf16(uint16_t* out, qrc_u64 n, qrc_u64 key, qrc_u64 offset, float sigma) {
    for (qrc_u64 i = (qrc_u64)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (qrc_u64)gridDim.x * blockDim.x)
        out[i] = qrc_gen::f32_to_bf16_rn(__fmul_rn(qrc_gen::normal01(key, offset + i), sigma));
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

namespace {

thread_local int g_last_cuda = 0;

#define QRC_CK(call)                                                      \
    do {                                                                  \
        cudaError_t e_ = (call);                                          \
        if (e_ != cudaSuccess) { g_last_cuda = (int)e_; return QRC_ERR_CUDA; } \
    } while (0)

// Makes `dev` current for the scope and restores the caller's device.  When
// `dev` is already current nothing is touched, so a context the caller made
// current through the driver API (as the QuickRunCUDA harness does with
// cuCtxCreate) stays current.
struct DeviceScope {
    int prev = -1;
    bool ok = false, switched = false;
    explicit DeviceScope(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev == dev) { ok = true; return; }
        ok = cudaSetDevice(dev) == cudaSuccess;
        switched = ok && prev >= 0;
    }
    ~DeviceScope() { if (switched) cudaSetDevice(prev); }
};

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

constexpr size_t kMapHeaderWords = qrc::O_PAGE_BITS;

}  // namespace

struct qrc_ctx {
    int device = 0;
    int num_sms = 0;
    int mode = QRC_MODE_SIDE_AWARE;
    int blocks_per_sm = 1;
    int threads = 1024;
    int bulk_slots = 0;             // 0: register loads; >= 2: bulk-copy staging slots per warp
    int overlap = 1;                // programmatic dependent launch of reductions
    int quant_side_aware = 1;       // side-aware quantize pass when the input is mapped
    int quant_fused = 1;            // single-launch fused quantize when its conditions hold
    int fused_checked = 0;          // 0 not yet, 1 the fused launch fits this device, -1 it does not
    const void* base = nullptr;
    size_t bytes = 0;
    qrc_u32* d_map = nullptr;
    size_t map_words = 0;
    qrc_side_info info{};
    float* d_scalars = nullptr;     // [0] amax scratch, [1] host-path result
    // host-buffer path (qrc_absmax_f32_host): staging buffer with its own side
    // map, a copy stream, one event and one partial result per chunk
    float* d_stage = nullptr;
    size_t stage_cap = 0;           // floats; 0 until qrc_host_reserve succeeded
    qrc_ctx* stage_ctx = nullptr;
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t entry_event = nullptr;
    std::vector<cudaEvent_t> chunk_events;
    float* d_partials = nullptr;    // one float per chunk
};

static void fill_info(qrc_ctx* c, const qrc_u32* h) {
    qrc_side_info& i = c->info;
    i.status = h[qrc::H_STATUS];
    i.mask = h[qrc::H_MASK];
    i.mask_measured = h[qrc::H_MASK_MEASURED];
    i.chunk_bytes = 1u << (h[qrc::H_CHUNK_LOG2] & 31u);
    i.num_sms_measured = h[qrc::H_NSM];
    i.sms_side0 = h[qrc::H_NSIDE0];
    i.sms_side1 = h[qrc::H_NSIDE1];
    i.num_pages = h[qrc::H_NPAGES];
    i.verify_probes = h[qrc::H_VERIFY_N];
    i.verify_mismatches = h[qrc::H_VERIFY_BAD];
    i.cal_lat_side0 = h[qrc::H_LAT0];
    i.cal_lat_side1 = h[qrc::H_LAT1];
    i.sm_lat_cluster0 = h[qrc::H_SM_C0];
    i.sm_lat_cluster1 = h[qrc::H_SM_C1];
    i.discover_smid = h[qrc::H_SMID_LAST];
}

// Dynamic shared memory of a launch: the bulk staging ring when enabled.
static size_t launch_smem(const qrc_ctx* c) {
    return c->bulk_slots ? (size_t)(c->threads / 32) * c->bulk_slots * qrc::kSlotStride : 0;
}

// Raises a kernel's dynamic shared memory limit on the current device to at
// least `smem` (launches above 48 KiB need it).  The attribute is per device,
// so what was granted is remembered per (kernel, device); thread-safe.
static cudaError_t grant_smem(const void* kernel, size_t smem) {
    if (smem <= 48 * 1024) return cudaSuccess;
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, size_t> granted;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    size_t& g = granted[{kernel, dev}];
    if (smem <= g) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) g = smem;
    return e;
}

template <int T>
static cudaError_t allow_smem(size_t smem) {
    cudaError_t e = grant_smem((const void*)qrc_k_absmax_f32<T>, smem);
    return e != cudaSuccess ? e : grant_smem((const void*)qrc_k_amax_bf16<T>, smem);
}

// Launches `kernel` with programmatic stream serialization when the context
// allows overlap: the kernel's CTAs may then be scheduled while the previous
// grid in the stream drains; the kernel itself waits (griddepcontrol.wait)
// before it touches anything the previous grid could still be using.
template <typename... KArgs, typename... Args>
static cudaError_t launch(const qrc_ctx* c, void (*kernel)(KArgs...), int grid, int block, size_t smem,
                          cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = c->overlap ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

static int launch_absmax(qrc_ctx* c, const float* in, size_t n, float* out, cudaStream_t s) {
    const int grid = c->num_sms * c->blocks_per_sm;
    const qrc_u32 mode = (qrc_u32)c->mode;
    const size_t smem = launch_smem(c);
    const qrc_u64 n64 = n;
    switch (c->threads) {
        case 1024: QRC_CK(allow_smem<1024>(smem)); QRC_CK(launch(c, qrc_k_absmax_f32<1024>, grid, 1024, smem, s, in, n64, c->d_map, out, mode)); break;
        case 512:  QRC_CK(allow_smem<512>(smem)); QRC_CK(launch(c, qrc_k_absmax_f32<512>, grid, 512, smem, s, in, n64, c->d_map, out, mode)); break;
        default:   QRC_CK(allow_smem<256>(smem)); QRC_CK(launch(c, qrc_k_absmax_f32<256>, grid, 256, smem, s, in, n64, c->d_map, out, mode)); break;
    }
    return QRC_OK;
}

QRC_API int qrc_ctx_create(qrc_ctx** out, int device, const void* d_base, size_t bytes, void* stream) {
    if (!out) return QRC_ERR_INVALID;
    *out = nullptr;
    if (d_base && ((uintptr_t)d_base & 3)) return QRC_ERR_INVALID;
    int ndev = 0;
    QRC_CK(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return QRC_ERR_DEVICE;
    DeviceScope scope(device);
    if (!scope.ok) return QRC_ERR_DEVICE;
    int major = 0, sms = 0;
    QRC_CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
    QRC_CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    if (major != 10) return QRC_ERR_DEVICE;

    qrc_ctx* c = new qrc_ctx();
    c->device = device;
    c->num_sms = sms;
    c->base = d_base;
    c->bytes = d_base ? bytes : 0;
    const uint64_t pages = d_base ? (((uintptr_t)d_base + bytes + qrc::kPage - 1) / qrc::kPage -
                                     (uintptr_t)d_base / qrc::kPage) : 0;
    size_t cap_words = (size_t)((pages + 31) / 32) + 1;
    if (cap_words < qrc::kDefaultPageWords) cap_words = qrc::kDefaultPageWords;
    c->map_words = kMapHeaderWords + cap_words;
    cudaStream_t s = as_stream(stream);
    int rc = QRC_OK;
    do {
        if (cudaMalloc(&c->d_map, c->map_words * 4) != cudaSuccess ||
            cudaMalloc(&c->d_scalars, 64) != cudaSuccess) { rc = QRC_ERR_CUDA; break; }
        if (cudaMemsetAsync(c->d_map, 0, c->map_words * 4, s) != cudaSuccess ||
            cudaMemsetAsync(c->d_scalars, 0, 64, s) != cudaSuccess) { rc = QRC_ERR_CUDA; break; }
        qrc_k_set_word<<<1, 1, 0, s>>>(c->d_map, qrc::H_PAGE_WORDS_CAP, (qrc_u32)cap_words);
        if (d_base) qrc_k_discover<<<sms, 1024, 0, s>>>(d_base, (qrc_u64)bytes, c->d_map);
        if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess) { rc = QRC_ERR_CUDA; break; }
        qrc_u32 h[256];
        if (cudaMemcpy(h, c->d_map, sizeof(h), cudaMemcpyDeviceToHost) != cudaSuccess) { rc = QRC_ERR_CUDA; break; }
        fill_info(c, h);
        if (!d_base) c->info.status = QRC_SIDE_NOT_RUN;
    } while (0);
    if (rc != QRC_OK) {
        g_last_cuda = (int)cudaGetLastError();
        if (c->d_map) cudaFree(c->d_map);
        if (c->d_scalars) cudaFree(c->d_scalars);
        delete c;
        return rc;
    }
    *out = c;
    return QRC_OK;
}

// Frees the host-buffer path's staging (buffer, its context, stream, events,
// partials) and marks it absent.
static void host_release(qrc_ctx* c) {
    if (c->stage_ctx) { qrc_ctx_destroy(c->stage_ctx); c->stage_ctx = nullptr; }
    if (c->d_stage) { cudaFree(c->d_stage); c->d_stage = nullptr; }
    if (c->d_partials) { cudaFree(c->d_partials); c->d_partials = nullptr; }
    for (cudaEvent_t e : c->chunk_events) cudaEventDestroy(e);
    c->chunk_events.clear();
    if (c->entry_event) { cudaEventDestroy(c->entry_event); c->entry_event = nullptr; }
    if (c->copy_stream) { cudaStreamDestroy(c->copy_stream); c->copy_stream = nullptr; }
    c->stage_cap = 0;
}

QRC_API int qrc_ctx_destroy(qrc_ctx* c) {
    if (!c) return QRC_OK;
    DeviceScope scope(c->device);
    host_release(c);
    if (c->d_map) cudaFree(c->d_map);
    if (c->d_scalars) cudaFree(c->d_scalars);
    delete c;
    return QRC_OK;
}

QRC_API int qrc_ctx_get_info(const qrc_ctx* c, qrc_side_info* info) {
    if (!c || !info) return QRC_ERR_INVALID;
    *info = c->info;
    return QRC_OK;
}

QRC_API int qrc_ctx_set_mode(qrc_ctx* c, int mode) {
    const int read_mode = mode & 0xF, sched = mode & ~0xF;
    if (!c || read_mode < QRC_MODE_SIDE_AWARE || read_mode > QRC_MODE_STREAM ||
        (sched != 0 && sched != QRC_SCHED_STATIC && sched != QRC_SCHED_QUEUE && sched != QRC_SCHED_BALANCED))
        return QRC_ERR_INVALID;
    c->mode = mode;
    if (c->stage_ctx) c->stage_ctx->mode = mode;
    return QRC_OK;
}

QRC_API int qrc_ctx_set_launch(qrc_ctx* c, int blocks_per_sm, int threads) {
    if (!c || (threads != 256 && threads != 512 && threads != 1024)) return QRC_ERR_INVALID;
    if (blocks_per_sm < 1 || blocks_per_sm * threads > 2048) return QRC_ERR_INVALID;
    if (c->bulk_slots && (blocks_per_sm != 1 || (size_t)(threads / 32) * c->bulk_slots * qrc::kSlotStride > 227 * 1024))
        return QRC_ERR_INVALID;
    c->blocks_per_sm = blocks_per_sm;
    c->threads = threads;
    if (c->stage_ctx) qrc_ctx_set_launch(c->stage_ctx, blocks_per_sm, threads);
    return QRC_OK;
}

QRC_API int qrc_ctx_set_pipeline(qrc_ctx* c, int slots) {
    if (!c || slots < 0 || slots == 1 || slots > 16) return QRC_ERR_INVALID;
    if (slots) {
        const size_t smem = (size_t)(c->threads / 32) * slots * qrc::kSlotStride;
        if (smem > 227 * 1024 || c->blocks_per_sm != 1) return QRC_ERR_INVALID;
    }
    c->bulk_slots = slots;
    if (c->stage_ctx) c->stage_ctx->bulk_slots = slots;
    return QRC_OK;
}

QRC_API int qrc_ctx_set_overlap(qrc_ctx* c, int enable) {
    if (!c || (enable != 0 && enable != 1)) return QRC_ERR_INVALID;
    c->overlap = enable;
    if (c->stage_ctx) c->stage_ctx->overlap = enable;
    return QRC_OK;
}

QRC_API int qrc_absmax_f32(const float* d_in, size_t n, float* d_out, qrc_ctx* c, void* stream) {
    if (!c || !d_out || (n && !d_in) || ((uintptr_t)d_in & 3)) return QRC_ERR_INVALID;
    if (n > ((size_t)1 << 61)) return QRC_ERR_RANGE;
    DeviceScope scope(c->device);
    if (!scope.ok) return QRC_ERR_STATE;
    return launch_absmax(c, d_in, n, d_out, as_stream(stream));
}

template <class Op, int T>
static cudaError_t launch_reduce_t(qrc_ctx* c, const float* in, qrc_u64 n, void* out, size_t smem, cudaStream_t s) {
    const cudaError_t e = grant_smem((const void*)qrc_k_reduce_f32<Op, T>, smem);
    if (e != cudaSuccess) return e;
    return launch(c, qrc_k_reduce_f32<Op, T>, c->num_sms * c->blocks_per_sm, T, smem, s, in, n, c->d_map, out,
                  (qrc_u32)c->mode);
}

template <class Op>
static int launch_reduce(qrc_ctx* c, const float* in, size_t n, void* out, cudaStream_t s) {
    const size_t smem = launch_smem(c);
    switch (c->threads) {
        case 1024: QRC_CK((launch_reduce_t<Op, 1024>(c, in, n, out, smem, s))); break;
        case 512:  QRC_CK((launch_reduce_t<Op, 512>(c, in, n, out, smem, s))); break;
        default:   QRC_CK((launch_reduce_t<Op, 256>(c, in, n, out, smem, s))); break;
    }
    return QRC_OK;
}

QRC_API int qrc_reduce_f32(const float* d_in, size_t n, int op, void* d_out, qrc_ctx* c, void* stream) {
    if (!c || !d_out || (n && !d_in) || ((uintptr_t)d_in & 3)) return QRC_ERR_INVALID;
    if (op < QRC_OP_ABSMAX || op > QRC_OP_SUMSQ) return QRC_ERR_INVALID;
    if (op >= QRC_OP_SUM && ((uintptr_t)d_out & 7)) return QRC_ERR_INVALID;
    if (n > ((size_t)1 << 61)) return QRC_ERR_RANGE;
    DeviceScope scope(c->device);
    if (!scope.ok) return QRC_ERR_STATE;
    cudaStream_t s = as_stream(stream);
    switch (op) {
        case QRC_OP_ABSMAX: return launch_absmax(c, d_in, n, (float*)d_out, s);
        case QRC_OP_MAX: return launch_reduce<qrc::OpMaxF32>(c, d_in, n, d_out, s);
        case QRC_OP_MIN: return launch_reduce<qrc::OpMinF32>(c, d_in, n, d_out, s);
        case QRC_OP_SUM: return launch_reduce<qrc::OpSumF32>(c, d_in, n, d_out, s);
        default: return launch_reduce<qrc::OpSumSqF32>(c, d_in, n, d_out, s);
    }
}

// ---------------------------------------------------------------------------
// Cross-GPU exchange (one rank per GPU)
// ---------------------------------------------------------------------------

struct qrc_xchg {
    int device = 0, rank = 0, world = 1;
    qrc_u64* d_slots = nullptr;             // 2 x world words, zeroed
    qrc_u64** d_peers = nullptr;            // world pointers, on the device
    qrc_u64* h_peers[QRC_XCHG_MAX_WORLD] = {};
    bool opened[QRC_XCHG_MAX_WORLD] = {};   // IPC mappings to close
    qrc_u32 epoch = 0;
};

QRC_API int qrc_xchg_create(qrc_xchg** out, int device, int rank, int world) {
    if (!out || world < 1 || world > QRC_XCHG_MAX_WORLD || rank < 0 || rank >= world) return QRC_ERR_INVALID;
    *out = nullptr;
    DeviceScope scope(device);
    if (!scope.ok) return QRC_ERR_DEVICE;
    qrc_xchg* x = new qrc_xchg();
    x->device = device; x->rank = rank; x->world = world;
    if (cudaMalloc(&x->d_slots, 2 * (size_t)world * sizeof(qrc_u64)) != cudaSuccess ||
        cudaMalloc(&x->d_peers, (size_t)world * sizeof(qrc_u64*)) != cudaSuccess ||
        cudaMemset(x->d_slots, 0, 2 * (size_t)world * sizeof(qrc_u64)) != cudaSuccess) {
        g_last_cuda = (int)cudaGetLastError();
        if (x->d_slots) cudaFree(x->d_slots);
        if (x->d_peers) cudaFree(x->d_peers);
        delete x;
        return QRC_ERR_CUDA;
    }
    x->h_peers[rank] = x->d_slots;
    *out = x;
    return QRC_OK;
}

QRC_API int qrc_xchg_get_handle(const qrc_xchg* x, void* handle) {
    if (!x || !handle) return QRC_ERR_INVALID;
    DeviceScope scope(x->device);
    if (!scope.ok) return QRC_ERR_DEVICE;
    cudaIpcMemHandle_t h;
    QRC_CK(cudaIpcGetMemHandle(&h, x->d_slots));
    static_assert(sizeof(h) == QRC_XCHG_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle, &h, sizeof(h));
    return QRC_OK;
}

static int xchg_set(qrc_xchg* x, int peer, qrc_u64* p, bool opened) {
    x->h_peers[peer] = p;
    x->opened[peer] = opened;
    QRC_CK(cudaMemcpy(x->d_peers, x->h_peers, (size_t)x->world * sizeof(qrc_u64*), cudaMemcpyHostToDevice));
    return QRC_OK;
}

QRC_API int qrc_xchg_set_peer(qrc_xchg* x, int peer, const void* handle) {
    if (!x || !handle || peer < 0 || peer >= x->world || peer == x->rank || x->h_peers[peer]) return QRC_ERR_INVALID;
    DeviceScope scope(x->device);
    if (!scope.ok) return QRC_ERR_DEVICE;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    QRC_CK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    return xchg_set(x, peer, (qrc_u64*)p, true);
}

QRC_API int qrc_xchg_debug_set_peer_ptr(qrc_xchg* x, int peer, void* d_slots) {
    if (!x || !d_slots || peer < 0 || peer >= x->world || peer == x->rank || x->h_peers[peer]) return QRC_ERR_INVALID;
    DeviceScope scope(x->device);
    if (!scope.ok) return QRC_ERR_DEVICE;
    return xchg_set(x, peer, (qrc_u64*)d_slots, false);
}

QRC_API void* qrc_xchg_debug_slots(const qrc_xchg* x) { return x ? (void*)x->d_slots : nullptr; }

QRC_API int qrc_xchg_debug_post(qrc_xchg* x, int peer, uint32_t epoch, uint32_t value_bits) {
    if (!x || peer < 0 || peer >= x->world) return QRC_ERR_INVALID;
    DeviceScope scope(x->device);
    if (!scope.ok) return QRC_ERR_DEVICE;
    const qrc_u64 word = ((qrc_u64)epoch << 32) | value_bits;
    QRC_CK(cudaMemcpy(x->d_slots + (size_t)(epoch & 1u) * x->world + peer, &word, sizeof(word),
                      cudaMemcpyHostToDevice));
    return QRC_OK;
}
QRC_API uint32_t qrc_xchg_epoch(const qrc_xchg* x) { return x ? x->epoch : 0u; }

QRC_API int qrc_xchg_destroy(qrc_xchg* x) {
    if (!x) return QRC_OK;
    DeviceScope scope(x->device);
    for (int p = 0; p < x->world; p++)
        if (x->opened[p]) cudaIpcCloseMemHandle(x->h_peers[p]);
    if (x->d_slots) cudaFree(x->d_slots);
    if (x->d_peers) cudaFree(x->d_peers);
    delete x;
    return QRC_OK;
}

QRC_API int qrc_absmax_f32_allreduce(const float* d_in, size_t n, float* d_out, qrc_ctx* c, qrc_xchg* x,
                                     void* stream) {
    if (!c || !x || !d_out || (n && !d_in) || ((uintptr_t)d_in & 3)) return QRC_ERR_INVALID;
    if (x->device != c->device) return QRC_ERR_INVALID;
    if (n > ((size_t)1 << 61)) return QRC_ERR_RANGE;
    for (int p = 0; p < x->world; p++)
        if (!x->h_peers[p]) return QRC_ERR_STATE;            // a peer's slots are not mapped yet
    DeviceScope scope(c->device);
    if (!scope.ok) return QRC_ERR_STATE;
    cudaStream_t s = as_stream(stream);
    const qrc::XchgArgs xa{x->d_slots, x->d_peers, (qrc_u32)x->rank, (qrc_u32)x->world, ++x->epoch};
    const int grid = c->num_sms * c->blocks_per_sm;
    const size_t smem = launch_smem(c);
    const qrc_u32 mode = (qrc_u32)c->mode;
    switch (c->threads) {
        case 1024:
            QRC_CK(grant_smem((const void*)qrc_k_absmax_f32_xchg<1024>, smem));
            QRC_CK(launch(c, qrc_k_absmax_f32_xchg<1024>, grid, 1024, smem, s, d_in, (qrc_u64)n, c->d_map, d_out, mode, xa));
            break;
        case 512:
            QRC_CK(grant_smem((const void*)qrc_k_absmax_f32_xchg<512>, smem));
            QRC_CK(launch(c, qrc_k_absmax_f32_xchg<512>, grid, 512, smem, s, d_in, (qrc_u64)n, c->d_map, d_out, mode, xa));
            break;
        default:
            QRC_CK(grant_smem((const void*)qrc_k_absmax_f32_xchg<256>, smem));
            QRC_CK(launch(c, qrc_k_absmax_f32_xchg<256>, grid, 256, smem, s, d_in, (qrc_u64)n, c->d_map, d_out, mode, xa));
            break;
    }
    return QRC_OK;
}

// Host-buffer path: the input crosses PCIe in chunks of kHostChunkFloats on a
// copy stream, and each chunk is reduced on the caller's stream as soon as it
// has landed, so the reduction hides under the copy of the next chunk; one
// small kernel then takes the maximum of the per-chunk results.
constexpr size_t kHostChunkFloats = 64ull << 20;          // 256 MiB: 128 whole 2 MiB pages

// Maximum of `k` per-chunk results.  An unsigned maximum of the bit patterns:
// the results are non-negative floats or NaN (a reduction whose bounded wait
// gave up), and the NaN pattern 0x7FFFFFFF orders above every one of them.
__global__ void qrc_k_max_partials(const float* partials, qrc_u32 k, float* out) {
    qrc_u32 m = 0;
    for (qrc_u32 i = threadIdx.x; i < k; i += blockDim.x) {
        const qrc_u32 b = __float_as_uint(partials[i]);
        m = b > m ? b : m;
    }
    m = qrc::block_max(m);
    if (threadIdx.x == 0) *out = __uint_as_float(m);
}

QRC_API int qrc_host_reserve(qrc_ctx* c, size_t n) {
    if (!c) return QRC_ERR_INVALID;
    if (n > ((size_t)1 << 61)) return QRC_ERR_RANGE;
    if (n <= c->stage_cap) return QRC_OK;
    DeviceScope scope(c->device);
    if (!scope.ok) return QRC_ERR_STATE;
    host_release(c);                                       // capacity stays 0 until all of it exists
    const size_t chunks = (n + kHostChunkFloats - 1) / kHostChunkFloats;
    int rc = QRC_OK;
    do {
        if (cudaMalloc(&c->d_stage, n * sizeof(float)) != cudaSuccess ||
            cudaMalloc(&c->d_partials, chunks * sizeof(float)) != cudaSuccess ||
            cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->entry_event, cudaEventDisableTiming) != cudaSuccess) {
            rc = QRC_ERR_CUDA; break;
        }
        c->chunk_events.reserve(chunks);
        for (size_t i = 0; i < chunks && rc == QRC_OK; i++) {
            cudaEvent_t e;
            if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) rc = QRC_ERR_CUDA;
            else c->chunk_events.push_back(e);
        }
        if (rc != QRC_OK) break;
        rc = qrc_ctx_create(&c->stage_ctx, c->device, c->d_stage, n * sizeof(float), nullptr);
    } while (0);
    if (rc != QRC_OK) {
        if (rc == QRC_ERR_CUDA && g_last_cuda == 0) g_last_cuda = (int)cudaGetLastError();
        host_release(c);
        return rc;
    }
    c->stage_ctx->mode = c->mode;
    c->stage_ctx->blocks_per_sm = c->blocks_per_sm;
    c->stage_ctx->threads = c->threads;
    c->stage_ctx->bulk_slots = c->bulk_slots;
    c->stage_ctx->overlap = c->overlap;
    c->stage_cap = n;
    return QRC_OK;
}

QRC_API int qrc_absmax_f32_host(const float* h_in, size_t n, float* h_out, qrc_ctx* c, void* stream) {
    if (!c || !h_out || (n && !h_in)) return QRC_ERR_INVALID;
    if (n > ((size_t)1 << 61)) return QRC_ERR_RANGE;
    DeviceScope scope(c->device);
    if (!scope.ok) return QRC_ERR_STATE;
    cudaStream_t s = as_stream(stream);
    if (n == 0) { *h_out = 0.0f; return QRC_OK; }
    const int rr = qrc_host_reserve(c, n);
    if (rr != QRC_OK) return rr;
    qrc_ctx* sc = c->stage_ctx;
    const size_t chunks = (n + kHostChunkFloats - 1) / kHostChunkFloats;
    // The copies start after everything the caller queued on `stream` before
    // this call (which may still be producing h_in, or reading the staging).
    QRC_CK(cudaEventRecord(c->entry_event, s));
    QRC_CK(cudaStreamWaitEvent(c->copy_stream, c->entry_event, 0));
    for (size_t i = 0; i < chunks; i++) {
        const size_t off = i * kHostChunkFloats, len = n - off < kHostChunkFloats ? n - off : kHostChunkFloats;
        QRC_CK(cudaMemcpyAsync(c->d_stage + off, h_in + off, len * sizeof(float), cudaMemcpyHostToDevice,
                               c->copy_stream));
        QRC_CK(cudaEventRecord(c->chunk_events[i], c->copy_stream));
    }
    for (size_t i = 0; i < chunks; i++) {
        const size_t off = i * kHostChunkFloats, len = n - off < kHostChunkFloats ? n - off : kHostChunkFloats;
        QRC_CK(cudaStreamWaitEvent(s, c->chunk_events[i], 0));
        const int rc = launch_absmax(sc, c->d_stage + off, len, c->d_partials + i, s);
        if (rc != QRC_OK) return rc;
    }
    qrc_k_max_partials<<<1, 256, 0, s>>>(c->d_partials, (qrc_u32)chunks, c->d_scalars + 1);
    QRC_CK(cudaGetLastError());
    QRC_CK(cudaMemcpyAsync(h_out, c->d_scalars + 1, sizeof(float), cudaMemcpyDeviceToHost, s));
    QRC_CK(cudaStreamSynchronize(s));
    return QRC_OK;
}

// Whether the single-launch fused quantize can run: the input inside the
// context's side-aware buffer, vector-aligned, every SM labelled by discovery
// (each SM gets exactly one CTA, so every static share is read once), and
// exactly one 1024-thread CTA with the stash's shared memory fits per SM, so
// a grid of one CTA per SM is resident at once.
static bool fused_quant_ok(qrc_ctx* c, const uint16_t* d_in, size_t n, const uint8_t* d_q) {
    if (!c->quant_fused || !n || n > ((size_t)1 << 46)) return false;   // 32-bit block indices in the kernel
    const bool mapped = c->info.status == QRC_SIDE_OK && (uintptr_t)d_in >= (uintptr_t)c->base &&
                        (uintptr_t)d_in + 2 * n <= (uintptr_t)c->base + c->bytes &&
                        c->info.chunk_bytes == 4096 && c->mode != QRC_MODE_STREAM;
    const bool aligned = ((uintptr_t)d_in & 15) == 0 && ((uintptr_t)d_q & 7) == 0;
    const qrc_side_info& i = c->info;
    if (!mapped || !aligned || i.num_sms_measured != (uint32_t)c->num_sms ||
        i.sms_side0 + i.sms_side1 != (uint32_t)c->num_sms || i.sms_side0 > 128 || i.sms_side1 > 128)
        return false;
    if (c->fused_checked == 0) {
        int per_sm = 0;
        bool ok = grant_smem((const void*)qrc_k_amax_quant_fused, kFusedSmemBytes) == cudaSuccess &&
                  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qrc_k_amax_quant_fused, 1024,
                                                                kFusedSmemBytes) == cudaSuccess && per_sm == 1;
        cudaGetLastError();
        c->fused_checked = ok ? 1 : -1;
    }
    return c->fused_checked > 0;
}

QRC_API int qrc_amax_quant_e4m3(const uint16_t* d_in, size_t n, uint8_t* d_q, float* d_scale,
                                float* d_amax, qrc_ctx* c, void* stream) {
    if (!c || !d_scale || (n && (!d_in || !d_q)) || ((uintptr_t)d_in & 1)) return QRC_ERR_INVALID;
    DeviceScope scope(c->device);
    if (!scope.ok) return QRC_ERR_STATE;
    cudaStream_t s = as_stream(stream);
    float* amax = d_amax ? d_amax : c->d_scalars;
    const qrc_u64 n64 = n;
    const qrc_u32 mode = (qrc_u32)c->mode;
    if (fused_quant_ok(c, d_in, n, d_q)) {
        // One CTA per SM: fused_quant_ok checked that exactly one fits and that
        // discovery saw every SM, so all CTAs are resident together (its grid
        // barrier relies on that; the wait is bounded all the same).  Not a
        // cooperative launch: the runtime gives those no programmatic
        // overlap with the previous kernel, which costs about 5 us a launch.
        QRC_CK(launch(c, qrc_k_amax_quant_fused, c->num_sms, 1024, kFusedSmemBytes, s, d_in, n64, d_q, amax, d_scale,
                      c->d_map, mode));
        return QRC_OK;
    }
    const int grid = c->num_sms * c->blocks_per_sm;
    const size_t smem = launch_smem(c);
    switch (c->threads) {
        case 1024: QRC_CK(allow_smem<1024>(smem)); QRC_CK(launch(c, qrc_k_amax_bf16<1024>, grid, 1024, smem, s, d_in, n64, c->d_map, amax, d_scale, mode)); break;
        case 512:  QRC_CK(allow_smem<512>(smem)); QRC_CK(launch(c, qrc_k_amax_bf16<512>, grid, 512, smem, s, d_in, n64, c->d_map, amax, d_scale, mode)); break;
        default:   QRC_CK(allow_smem<256>(smem)); QRC_CK(launch(c, qrc_k_amax_bf16<256>, grid, 256, smem, s, d_in, n64, c->d_map, amax, d_scale, mode)); break;
    }
    // The side-aware pass needs the input inside the context's mapped buffer
    // (the same test the amax pass makes on the device) and vector alignment.
    const bool mapped = c->info.status == QRC_SIDE_OK && (uintptr_t)d_in >= (uintptr_t)c->base &&
                        (uintptr_t)d_in + 2 * n <= (uintptr_t)c->base + c->bytes &&
                        c->info.chunk_bytes == 4096 && c->mode != QRC_MODE_STREAM;
    const bool aligned = ((uintptr_t)d_in & 15) == 0 && ((uintptr_t)d_q & 7) == 0;
    if (n && mapped && aligned && c->quant_side_aware)
        QRC_CK(launch(c, qrc_k_quant_e4m3_sa, c->num_sms, 1024, 0, s, d_in, n64, d_q, (const float*)d_scale,
                      c->d_map, mode));
    else if (n)
        QRC_CK(launch(c, qrc_k_quant_e4m3, c->num_sms * 2, 512, 0, s, d_in, n64, d_q, (const float*)d_scale));
    return QRC_OK;
}

QRC_API int qrc_debug_quant_launches(qrc_ctx* c, const uint16_t* d_in, size_t n, const uint8_t* d_q) {
    if (!c) return QRC_ERR_INVALID;
    DeviceScope scope(c->device);
    if (!scope.ok) return QRC_ERR_STATE;
    if (!n) return 1;
    return fused_quant_ok(c, d_in, n, d_q) ? 1 : 2;
}

QRC_API int qrc_ctx_debug_quant_fused(qrc_ctx* c, int enable) {
    if (!c) return QRC_ERR_INVALID;
    c->quant_fused = enable ? 1 : 0;
    return QRC_OK;
}

// ---- generators ------------------------------------------------------------

static int fill_grid(void) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms * 8;
}

QRC_API int qrc_fill_uniform_f32(float* d_out, size_t n, uint64_t seed, uint64_t offset, void* stream) {
    if (n && !d_out) return QRC_ERR_INVALID;
    if (!n) return QRC_OK;
    qrc_k_fill_uniform<<<fill_grid(), 256, 0, as_stream(stream)>>>(d_out, n, qrc_gen::key_of(seed), offset);
    QRC_CK(cudaGetLastError());
    return QRC_OK;
}

QRC_API int qrc_fill_normal_f32(float* d_out, size_t n, uint64_t seed, uint64_t offset, float sigma, void* stream) {
    if (n && !d_out) return QRC_ERR_INVALID;
    if (!n) return QRC_OK;
    qrc_k_fill_normal<<<fill_grid(), 256, 0, as_stream(stream)>>>(d_out, n, qrc_gen::key_of(seed), offset, sigma);
    QRC_CK(cudaGetLastError());
    return QRC_OK;
}

QRC_API int qrc_fill_normal_bf16(uint16_t* d_out, size_t n, uint64_t seed, uint64_t offset, float sigma, void* stream) {
    if (n && !d_out) return QRC_ERR_INVALID;
    if (!n) return QRC_OK;
    qrc_k_fill_normal_bf16<<<fill_grid(), 256, 0, as_stream(stream)>>>(d_out, n, qrc_gen::key_of(seed), offset, sigma);
    QRC_CK(cudaGetLastError());
    return QRC_OK;
}

QRC_API int qrc_host_fill_uniform_f32(float* h_out, size_t n, uint64_t seed, uint64_t offset) {
    if (n && !h_out) return QRC_ERR_INVALID;
    const uint64_t key = qrc_gen::key_of(seed);
    #pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) h_out[i] = qrc_gen::uniform_pm1(key, offset + i);
    return QRC_OK;
}

QRC_API int qrc_host_fill_normal_f32(float* h_out, size_t n, uint64_t seed, uint64_t offset, float sigma) {
    if (n && !h_out) return QRC_ERR_INVALID;
    const uint64_t key = qrc_gen::key_of(seed);
    #pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) h_out[i] = qrc_gen::normal01(key, offset + i) * sigma;
    return QRC_OK;
}

QRC_API uint64_t qrc_outlier_index(uint64_t seed, uint64_t n) { return qrc_gen::outlier_index(seed, n); }
QRC_API int qrc_outlier_sign(uint64_t seed) { return qrc_gen::outlier_sign(seed); }

// ---- strings, version, diagnostics -------------------------------------------

QRC_API const char* qrc_status_string(int st) {
    switch (st) {
        case QRC_OK: return "ok";
        case QRC_ERR_INVALID: return "invalid argument";
        case QRC_ERR_CUDA: return "CUDA runtime error";
        case QRC_ERR_DEVICE: return "no such sm_100 device";
        case QRC_ERR_RANGE: return "input too large";
        case QRC_ERR_STATE: return "context used on another device";
        default: return "unknown status";
    }
}

QRC_API const char* qrc_side_status_string(uint32_t st) {
    switch (st) {
        case QRC_SIDE_OK: return "side-aware";
        case QRC_SIDE_TOO_SMALL: return "buffer holds no full 2 MiB page";
        case QRC_SIDE_NO_SM_SPLIT: return "SM latencies did not split into two sides";
        case QRC_SIDE_NO_HASH: return "no in-page address bit changed the side";
        case QRC_SIDE_BAD_HASH: return "hash granule below 512 bytes";
        case QRC_SIDE_NO_CAL_SPLIT: return "calibration words not separable";
        case QRC_SIDE_VERIFY_FAILED: return "side map failed verification";
        case QRC_SIDE_TOO_MANY_PAGES: return "too many pages for the map";
        case QRC_SIDE_UNALIGNED: return "buffer not 4-byte aligned";
        case QRC_SIDE_NOT_RUN: return "no buffer given: side-agnostic";
        default: return "unknown side status";
    }
}

QRC_API int qrc_last_cuda_error(void) { return g_last_cuda; }
QRC_API int qrc_version(void) { return 10000; }

QRC_API int qrc_ctx_read_map(const qrc_ctx* c, uint32_t* h, size_t words, size_t* total) {
    if (!c || (words && !h)) return QRC_ERR_INVALID;
    if (total) *total = c->map_words;
    if (words > c->map_words) words = c->map_words;
    DeviceScope scope(c->device);
    QRC_CK(cudaDeviceSynchronize());
    if (words) QRC_CK(cudaMemcpy(h, c->d_map, words * 4, cudaMemcpyDeviceToHost));
    return QRC_OK;
}

QRC_API int qrc_ctx_clear_diagnostics(qrc_ctx* c) {
    if (!c) return QRC_ERR_INVALID;
    DeviceScope scope(c->device);
    QRC_CK(cudaDeviceSynchronize());
    QRC_CK(cudaMemset(c->d_map + qrc::H_ERR, 0, 8 * 4));
    QRC_CK(cudaMemset(c->d_map + qrc::H_XCHG_ERR, 0, 4));
    return QRC_OK;
}

QRC_API int qrc_is_checked_build(void) {
#ifdef QRC_CHECKED
    return 1;
#else
    return 0;
#endif
}

QRC_API int qrc_debug_cvt_e4m3(const float* d_in, size_t n, uint8_t* d_out, void* stream) {
    if (n && (!d_in || !d_out)) return QRC_ERR_INVALID;
    if (!n) return QRC_OK;
    qrc_k_debug_cvt_e4m3<<<fill_grid(), 256, 0, as_stream(stream)>>>(d_in, n, d_out);
    QRC_CK(cudaGetLastError());
    return QRC_OK;
}

QRC_API int qrc_debug_read_stream(const void* d_in, size_t bytes, int depth, int threads, int blocks_per_sm,
                                  uint32_t* d_sink, void* stream) {
    if ((bytes && !d_in) || !d_sink || ((uintptr_t)d_in & 15)) return QRC_ERR_INVALID;
    int dev = 0, sms = 0;
    QRC_CK(cudaGetDevice(&dev));
    QRC_CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const qrc_u64 nv = bytes / 16;
    const int grid = sms * blocks_per_sm;
    cudaStream_t s = as_stream(stream);
    const uint4* p = (const uint4*)d_in;
    if (depth == 8 && threads == 1024 && blocks_per_sm == 1)
        qrc_k_read_stream<8, 1024, 1><<<grid, 1024, 0, s>>>(p, nv, d_sink);
    else if (depth == 4 && threads == 1024 && blocks_per_sm == 2)
        qrc_k_read_stream<4, 1024, 2><<<grid, 1024, 0, s>>>(p, nv, d_sink);
    else if (depth == 16 && threads == 512 && blocks_per_sm == 1)
        qrc_k_read_stream<16, 512, 1><<<grid, 512, 0, s>>>(p, nv, d_sink);
    else if (depth == 32 && threads == 256 && blocks_per_sm == 1)
        qrc_k_read_stream<32, 256, 1><<<grid, 256, 0, s>>>(p, nv, d_sink);
    else
        return QRC_ERR_INVALID;
    QRC_CK(cudaGetLastError());
    return QRC_OK;
}

QRC_API void* qrc_ctx_map_device_ptr(const qrc_ctx* c) { return c ? (void*)c->d_map : nullptr; }

QRC_API int qrc_ctx_debug_quant_side_aware(qrc_ctx* c, int enable) {
    if (!c) return QRC_ERR_INVALID;
    c->quant_side_aware = enable ? 1 : 0;
    return QRC_OK;
}

// ---------------------------------------------------------------------------
// Output buffers homed like an input (VMM)
// ---------------------------------------------------------------------------
// The die that homes an address is parity(addr & mask) ^ (a bit per physical
// 2 MiB page).  With the driver's virtual memory management the buffer is
// built page by page: physical 2 MiB pages are created in batches, mapped
// side by side and classified by a discovery run, and for every 2 MiB slot of
// the input's context the buffer maps a page whose bit matches.  The buffer
// keeps the input's offset within its first page, so equal offsets land on
// the same die.  Driver entry points come from cudaGetDriverEntryPoint: the
// library does not link libcuda.

namespace {
typedef CUresult (*PFN_gran)(size_t*, const CUmemAllocationProp*, CUmemAllocationGranularity_flags);
typedef CUresult (*PFN_create)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*, unsigned long long);
typedef CUresult (*PFN_release)(CUmemGenericAllocationHandle);
typedef CUresult (*PFN_reserve)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long);
typedef CUresult (*PFN_addrfree)(CUdeviceptr, size_t);
typedef CUresult (*PFN_map)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
typedef CUresult (*PFN_unmap)(CUdeviceptr, size_t);
typedef CUresult (*PFN_access)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t);

struct Vmm {
    PFN_gran gran = nullptr; PFN_create create = nullptr; PFN_release release = nullptr;
    PFN_reserve reserve = nullptr; PFN_addrfree addrfree = nullptr; PFN_map map = nullptr;
    PFN_unmap unmap = nullptr; PFN_access access = nullptr;
    bool load() {
        auto get = [](const char* name, void** fn) {
            cudaDriverEntryPointQueryResult q;
            return cudaGetDriverEntryPoint(name, fn, cudaEnableDefault, &q) == cudaSuccess &&
                   q == cudaDriverEntryPointSuccess && *fn;
        };
        return get("cuMemGetAllocationGranularity", (void**)&gran) && get("cuMemCreate", (void**)&create) &&
               get("cuMemRelease", (void**)&release) && get("cuMemAddressReserve", (void**)&reserve) &&
               get("cuMemAddressFree", (void**)&addrfree) && get("cuMemMap", (void**)&map) &&
               get("cuMemUnmap", (void**)&unmap) && get("cuMemSetAccess", (void**)&access);
    }
};
constexpr size_t kVmmPage = 2ull << 20;
constexpr int kVmmRounds = 8;                 // probe rounds, plus one per kVmmMaxProbe pages of input
constexpr size_t kVmmMaxProbe = 8192;         // candidate pages per round (16 GiB held at most)

std::vector<qrc_u32> read_words(const qrc_ctx* c, size_t first, size_t n) {
    std::vector<qrc_u32> w(n);
    if (cudaMemcpy(w.data(), c->d_map + first, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) w.clear();
    return w;
}
}  // namespace

struct qrc_vmm_buf {
    int device = 0;
    CUdeviceptr va = 0;
    size_t va_bytes = 0;
    std::vector<CUmemGenericAllocationHandle> pages;   // mapped, one per 2 MiB slot
    Vmm d;
};

static void vmm_drop(Vmm& d, std::vector<CUmemGenericAllocationHandle>& hs) {
    for (auto h : hs) d.release(h);
    hs.clear();
}

QRC_API int qrc_free_like(qrc_vmm_buf* b) {
    if (!b) return QRC_OK;
    DeviceScope scope(b->device);
    cudaDeviceSynchronize();
    if (b->va) {
        b->d.unmap(b->va, b->va_bytes);
        b->d.addrfree(b->va, b->va_bytes);
    }
    vmm_drop(b->d, b->pages);
    delete b;
    return QRC_OK;
}

QRC_API int qrc_alloc_like(qrc_vmm_buf** out, void** d_ptr, const qrc_ctx* like) {
    if (!out || !d_ptr || !like || !like->base || !like->bytes) return QRC_ERR_INVALID;
    *out = nullptr; *d_ptr = nullptr;
    if (like->info.status != QRC_SIDE_OK) return QRC_ERR_STATE;
    DeviceScope scope(like->device);
    if (!scope.ok) return QRC_ERR_DEVICE;
    qrc_vmm_buf* b = new qrc_vmm_buf();
    b->device = like->device;
    Vmm& d = b->d;
    if (!d.load()) { delete b; return QRC_ERR_DEVICE; }
    CUmemAllocationProp prop = {};
    prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop.location.id = like->device;
    size_t gran = 0;
    if (d.gran(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_MINIMUM) != CUDA_SUCCESS || gran == 0 || kVmmPage % gran) {
        delete b; return QRC_ERR_DEVICE;
    }
    CUmemAccessDesc acc = {};
    acc.location = prop.location;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;

    // What the input looks like: its page bits, mask and SM labels.
    const uintptr_t base = (uintptr_t)like->base, page_base = base & ~(uintptr_t)(kVmmPage - 1);
    const size_t P = (base + like->bytes - page_base + kVmmPage - 1) / kVmmPage;
    const std::vector<qrc_u32> hdr = read_words(like, 0, qrc::O_PAGE_BITS + (P + 31) / 32);
    if (hdr.empty()) { delete b; return QRC_ERR_CUDA; }
    std::vector<int> want(P);
    for (size_t p = 0; p < P; p++) want[p] = (hdr[qrc::O_PAGE_BITS + p / 32] >> (p % 32)) & 1;

    std::vector<CUmemGenericAllocationHandle> have[2];
    size_t need[2] = {0, 0};
    for (size_t p = 0; p < P; p++) need[want[p]]++;
    int rc = QRC_OK;
    const int rounds = kVmmRounds + (int)(P / kVmmMaxProbe);
    for (int round = 0; round < rounds && (have[0].size() < need[0] || have[1].size() < need[1]); round++) {
        const size_t short0 = need[0] > have[0].size() ? need[0] - have[0].size() : 0;
        const size_t short1 = need[1] > have[1].size() ? need[1] - have[1].size() : 0;
        size_t K = 2 * (short0 > short1 ? short0 : short1) + 4;
        if (K > kVmmMaxProbe) K = kVmmMaxProbe;
        std::vector<CUmemGenericAllocationHandle> batch;
        std::vector<char> kept;
        CUdeviceptr sva = 0;
        size_t mapped = 0;                                // slots [0, mapped) of sva hold a page
        bool ok = d.reserve(&sva, K * kVmmPage, kVmmPage, 0, 0) == CUDA_SUCCESS;
        if (!ok) sva = 0;
        for (size_t i = 0; ok && i < K; i++) {
            CUmemGenericAllocationHandle h;
            ok = d.create(&h, kVmmPage, &prop, 0) == CUDA_SUCCESS;
            if (ok) {
                batch.push_back(h);
                kept.push_back(0);
                ok = d.map(sva + i * kVmmPage, kVmmPage, 0, h, 0) == CUDA_SUCCESS;
                if (ok) mapped = i + 1;
            }
        }
        ok = ok && d.access(sva, K * kVmmPage, &acc, 1) == CUDA_SUCCESS;
        qrc_ctx* probe = nullptr;
        if (ok) ok = qrc_ctx_create(&probe, like->device, (const void*)sva, K * kVmmPage, nullptr) == QRC_OK &&
                     probe->info.status == QRC_SIDE_OK && probe->info.mask == like->info.mask;
        if (ok) {
            const std::vector<qrc_u32> ph = read_words(probe, 0, qrc::O_PAGE_BITS + (K + 31) / 32);
            ok = !ph.empty();
            int agree = 0, differ = 0;                    // are the two maps' side labels swapped?
            for (int s = 0; ok && s < qrc::kMaxSm; s++) {
                const qrc_u32 l1 = hdr[qrc::O_SM_SIDE + s], l2 = ph[qrc::O_SM_SIDE + s];
                if (l1 && l2) (((l1 - 1) & 1) == ((l2 - 1) & 1) ? agree : differ)++;
            }
            const int flip = differ > agree;
            for (size_t i = 0; ok && i < K; i++) {
                const int bit = ((ph[qrc::O_PAGE_BITS + i / 32] >> (i % 32)) & 1) ^ flip;
                if (have[bit].size() < need[bit]) { have[bit].push_back(batch[i]); kept[i] = 1; }
            }
        }
        if (probe) qrc_ctx_destroy(probe);
        cudaDeviceSynchronize();
        if (sva) {
            if (mapped) d.unmap(sva, mapped * kVmmPage);
            d.addrfree(sva, K * kVmmPage);
        }
        for (size_t i = 0; i < batch.size(); i++) if (!kept[i]) d.release(batch[i]);
        if (!ok) { rc = QRC_ERR_CUDA; break; }
    }
    if (rc == QRC_OK && (have[0].size() < need[0] || have[1].size() < need[1])) rc = QRC_ERR_STATE;
    if (rc == QRC_OK) {
        b->va_bytes = P * kVmmPage;
        bool ok = d.reserve(&b->va, b->va_bytes, kVmmPage, 0, 0) == CUDA_SUCCESS;
        if (!ok) b->va = 0;
        size_t taken[2] = {0, 0};
        for (size_t p = 0; ok && p < P; p++) {
            const CUmemGenericAllocationHandle h = have[want[p]][taken[want[p]]++];
            ok = d.map(b->va + p * kVmmPage, kVmmPage, 0, h, 0) == CUDA_SUCCESS;
            if (ok) b->pages.push_back(h);
            else d.release(h);                              // taken but not mapped
        }
        ok = ok && d.access(b->va, b->va_bytes, &acc, 1) == CUDA_SUCCESS;
        // pages not taken (none, when all went well) go back
        for (int s = 0; s < 2; s++)
            for (size_t i = taken[s]; i < have[s].size(); i++) d.release(have[s][i]);
        if (!ok) {
            if (b->va) {
                if (!b->pages.empty()) d.unmap(b->va, b->pages.size() * kVmmPage);
                d.addrfree(b->va, b->va_bytes);
                b->va = 0;
            }
            vmm_drop(d, b->pages);
            rc = QRC_ERR_CUDA;
        }
    } else {
        vmm_drop(d, have[0]);
        vmm_drop(d, have[1]);
    }
    if (rc != QRC_OK) { delete b; return rc; }
    *out = b;
    *d_ptr = (void*)(b->va + (base - page_base));
    return QRC_OK;
}

QRC_API int qrc_copy_f32(const float* d_x, float* d_y, size_t n, qrc_ctx* c, void* stream) {
    if (!c || (n && (!d_x || !d_y))) return QRC_ERR_INVALID;
    DeviceScope scope(c->device);
    if (!scope.ok) return QRC_ERR_STATE;
    cudaStream_t s = as_stream(stream);
    if (!n) return QRC_OK;
    const bool mapped = c->info.status == QRC_SIDE_OK && (uintptr_t)d_x >= (uintptr_t)c->base &&
                        (uintptr_t)d_x + 4 * n <= (uintptr_t)c->base + c->bytes && c->info.chunk_bytes == 4096;
    const bool aligned = ((uintptr_t)d_x & 15) == 0 && ((uintptr_t)d_y & 15) == 0;
    const bool apart = (uintptr_t)d_y >= (uintptr_t)d_x + 4 * n || (uintptr_t)d_x >= (uintptr_t)d_y + 4 * n;
    if (d_x == d_y) return QRC_OK;                       // copying a range onto itself changes nothing
    if (!apart) return QRC_ERR_INVALID;                 // partial overlap has no defined result
    if (mapped && aligned && c->mode != QRC_MODE_STREAM)
        QRC_CK(launch(c, qrc_k_copy_f32_sa, c->num_sms, 1024, 0, s, d_x, (qrc_u64)n, d_y, c->d_map,
                      (qrc_u32)c->mode));
    else
        QRC_CK(cudaMemcpyAsync(d_y, d_x, 4 * n, cudaMemcpyDeviceToDevice, s));
    return QRC_OK;
}
