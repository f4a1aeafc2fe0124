// side_aware_b200.cu -- L2-side-aware FP32 absmax for B200 (sm_100a).
//
// A drop-in kernel file for the QuickRunCUDA harness: it exports the harness'
// plugin ABI (`init` + `kernel`, QuickRunCUDA.cpp:408-411 and :466-499), so
//
//   QuickRunCUDA -i -p -t 1024 -A 1000000000 -0 1000000000 -T 100 -P 4.0 -U GB/s side_aware_b200.cu
//
// runs it exactly like the reference's tests/side_aware.cu.  The file is
// self-contained (no includes) so that NVRTC can compile it with the harness'
// options; the C-ABI library (qrc_abi.cu) includes it with QRC_NO_PLUGIN_ABI
// defined and launches the same device code from its own entry points.
//
// Plugin arguments (same slots as the reference, side_aware.cu:72 and :257):
//   A        input floats (the harness allocates it with cuMemAlloc, so it is
//            2 MiB aligned; any 4-byte aligned pointer works here)
//   B        side map / scratch, zeroed by the harness before init
//            (QuickRunCUDA.cpp:461-463); layout below, about 20 KiB
//   C        C[0] receives absmax(A) after every `kernel` launch
//   arg0     number of floats (`-0`)
//   arg1     read mode (`-1`): 0 side-aware, 1 page bits ignored (the
//            reference's FORCE_RANDOM_SIDE ablation), 2 every chunk read from
//            the far side (FORCE_WRONG_SIDE), 3 side-agnostic grid-stride stream;
//            plus 16 to force static shares, 32 the side queues, 48 static
//            shares with a queued tail (default: chosen by size).
//            `-H '#define FORCE_RANDOM_SIDE'` / FORCE_WRONG_SIDE also work.
//
// How B200 is modelled (the reference's model, side_aware.cu:8-12, re-measured
// here by discovery rather than assumed):
//   * each physical address is homed in the L2 of one of the two dies ("sides");
//   * inside a 2 MiB page the side is parity(addr & mask) XOR a per-page bit,
//     where mask covers address bits 4..20 and its lowest set bit is the chunk
//     size C (4 KiB on GB200: mask 0x1EF000, side_aware.cu:49);
//   * so the two C-byte halves of every 2C-aligned "pair" sit on opposite sides.
//
// Discovery (`init`, once per allocation) -- replaces side_aware.cu:72-210:
//   phase 1  every CTA times a dependent chain of same-value atomicCAS on a
//            word of the first full 2 MiB page ("anchor"); the chain never
//            changes memory (CAS writes back the value it read), unlike the
//            reference's exchange-then-restore (side_aware.cu:58-65).
//   phase 2  the last CTA to arrive (atomic ticket after a fence):
//            - splits SMs into two latency clusters (1-D 2-means, not the mean
//              threshold of side_aware.cu:94-100); side 0 = near the anchor,
//              so labels are absolute rather than relative to whichever SM
//              finished last (fixes the unlabelled page bits of :176-180);
//            - probes anchor ^ (1<<b), b = 4..20, from 21 warps at once to find
//              the mask (side_aware.cu:125-157 did this serially);
//            - calibrates this SM's latency to a known side-0 and side-1 word,
//              then probes one word per 2 MiB page from 30 warps in parallel
//              (side_aware.cu:173-190 probed ~1,900 pages serially);
//            - verifies the model on 80 extra probes; if it mispredicts more
//              than 1 in 8 the map is marked unusable and the reduction runs
//              side-agnostic (still exact).
//   Every wait in discovery is a bounded dependent chain; nothing spins.
//
// Reduction (`kernel`) -- replaces side_aware.cu:257-395:
//   * any grid and any block size that is a multiple of 32 (the reference
//     needed exactly one 1024-thread block per SM, :266-269);
//   * each CTA reads its SM's side from the map; for every pair it reads the
//     C-byte half homed on its own side.  Both sides walk every pair, one half
//     each, so every byte is read exactly once whatever the map says -- the
//     map only decides locality, never coverage;
//   * work goes out as static per-SM shares of 64 KiB blocks (inputs up to
//     256 MiB), as static shares for 5/8 (1/8 above 1 GiB) with the rest
//     claimed block by block from a per-side queue (larger inputs), or as
//     one-pair grabs from the per-side queues (launch shapes the shares
//     cannot serve);
//   * per element max(acc, |x|) with IEEE maxNum semantics written in PTX
//     (NaN never wins, -0 -> +0, denormals kept even under -use_fast_math);
//     QRC_PLUGIN_OP selects max, min, sum or sum of squares instead;
//   * warp max with redux.sync.max.u32 on the (non-negative) float bits, one
//     smem step per block, one red.max per block, then a fenced ticket: the
//     last CTA moves the result to C[0] and resets accumulator and queues, so
//     back-to-back launches need no host work (fixes the unfenced
//     scratch-then-ticket order of side_aware.cu:371-374).

#ifndef QRC_SIDE_AWARE_B200_CU
#define QRC_SIDE_AWARE_B200_CU

typedef unsigned int qrc_u32;
typedef unsigned long long qrc_u64;

#define QRC_DEV static __device__ __forceinline__
#define QRC_MEMBER __device__ __forceinline__

namespace qrc {

constexpr qrc_u32 kMagic = 0x51525341u;         // 'QRSA'
constexpr qrc_u64 kPage = 2ull * 1024 * 1024;   // side bit granularity (2 MiB pages)
constexpr int kProbeIters = 32;                  // dependent atomics per latency probe
constexpr int kMaxSm = 256;
// Compile-time knobs (a kernel-file user can set them with the harness' -H,
// like the reference's own #defines):
//   QRC_MAX_GRAB   queue schedule: most pairs a warp takes per queue atomic
//                  (guided: grabs shrink to 1 pair as its side's queue empties)
//   QRC_LOAD_KIND  0 ld.global.v4, 1 ld.global.nc.L1::no_allocate.L2::256B.v4,
//                  2 as 1 plus L2::evict_first, 3 256-bit ld.global.nc.v8,
//                  4 ld.global.nc.L1::no_allocate.v4 (no L2 prefetch size)
#ifndef QRC_MAX_GRAB
#define QRC_MAX_GRAB 1
#endif
#ifndef QRC_LOAD_KIND
#define QRC_LOAD_KIND 1
#endif
//   QRC_STEAL      1: a warp whose side queue is empty continues on the other
//                  side's queue (far reads, only in the tail), so a die with
//                  fewer SMs does not leave the other one idle at the end
#ifndef QRC_STEAL
#define QRC_STEAL 1
#endif
//   QRC_STRIDE_LOG2  queue positions map to pairs through an interleave: a
//                  grab of QRC_MAX_GRAB positions covers pairs 2^this apart,
//                  and consecutive grabs (other warps) cover adjacent pairs,
//                  so all warps of a side work inside one compact window of
//                  memory at a time; 0 maps positions to pairs in order
#ifndef QRC_STRIDE_LOG2
#define QRC_STRIDE_LOG2 0
#endif
#ifndef QRC_TIMELINE
#define QRC_TIMELINE 0
#endif
//   QRC_FINISH     1: block maxima leave as red.max and one acquire-release
//                  ticket atomic; 0: atomicMax, fence, ticket, fence
#ifndef QRC_FINISH
#define QRC_FINISH 1
#endif
//   QRC_SHARES     1: the static and balanced schedules may use static
//                  per-SM shares (see reduce_run); 0: every pair goes through
//                  the side queues
#ifndef QRC_SHARES
#define QRC_SHARES 1
#endif
//   QRC_STATIC_EIGHTHS  balanced schedule: eighths of the pairs covered by
//                  static shares; the rest is claimed block by block from the
//                  side queues, which absorbs SMs that run slower than their
//                  share assumes
//   QRC_STATIC_EIGHTHS_LARGE  the same above QRC_LARGE_PAIRS pairs (1 GiB),
//                  where a smaller static part measured faster (0.3-1 % at
//                  4 GB) and below which it measured slower
#ifndef QRC_STATIC_EIGHTHS
#define QRC_STATIC_EIGHTHS 5
#endif
#ifndef QRC_STATIC_EIGHTHS_LARGE
#define QRC_STATIC_EIGHTHS_LARGE 1
#endif
#ifndef QRC_LARGE_PAIRS
#define QRC_LARGE_PAIRS 131072
#endif
//   QRC_STATIC_MAX_PAIRS  automatic schedule: static shares alone up to this
//                  many 8 KiB pairs, the balanced schedule above
//   QRC_PLAIN_MAX_BYTES  static shares of inputs up to this size are read
//                  with plain ld.global.v4 (flavour 0), larger ones with
//                  QRC_LOAD_KIND.  Back to back, plain loads keep much of an
//                  input up to ~1.1x the 126 MB L2 resident (112-128 MiB:
//                  11-11.8 TB/s against 7.0-7.3 TB/s; 136 MiB: +2 %); from
//                  144 MiB on they lose 17-21 % to the non-coherent path
#ifndef QRC_PLAIN_MAX_BYTES
#define QRC_PLAIN_MAX_BYTES (136ull << 20)
#endif
#ifndef QRC_STATIC_MAX_PAIRS
#define QRC_STATIC_MAX_PAIRS 32768
#endif
//   QRC_SM_FIRST_MAX_PAIRS  static shares of up to this many pairs (with no
//                  queued tail) hand
//                  consecutive 8-pair blocks to different SMs; larger ones
//                  give each SM G adjacent blocks (see Shares)
#ifndef QRC_SM_FIRST_MAX_PAIRS
#define QRC_SM_FIRST_MAX_PAIRS 16384
#endif
//   QRC_ACROSS     1: a warp takes its next 8 chunks together and loads slice k
//                  of all 8 before slice k+1 (8 chunks in flight, one 512-byte
//                  row of each); 0: one chunk at a time, all 8 rows
#ifndef QRC_ACROSS
#define QRC_ACROSS 0
#endif
//   QRC_TIMELINE   1: each CTA of a reduction records its start and end
//                  %globaltimer, side, SM and the chunks it read from the other
//                  side's queue in the map (words O_TIMELINE + 4*CTA, up to
//                  256 CTAs); word O_TIMELINE + 1023 gets the time the last CTA
//                  published, + 1022 the previous launch's; diagnostics, off by
//                  default
constexpr qrc_u32 kMaxGrab = QRC_MAX_GRAB;
constexpr int kStrideLog2 = QRC_STRIDE_LOG2;
static_assert((QRC_MAX_GRAB & (QRC_MAX_GRAB - 1)) == 0, "QRC_MAX_GRAB must be a power of two");
constexpr int kGrabLog2 = QRC_MAX_GRAB >= 16 ? 4 : QRC_MAX_GRAB >= 8 ? 3 : QRC_MAX_GRAB >= 4 ? 2 : QRC_MAX_GRAB >= 2 ? 1 : 0;
constexpr int kVerifyRandom = 64;
constexpr int kVerifyCal = 8;                    // anchor + partner re-probes in verification
constexpr int kCalProbes = 16;                   // per side, calibration wave
constexpr int kDiagPages = 1024;                 // raw page latencies kept for diagnostics
constexpr qrc_u32 kDefaultPageWords = 1024;      // page-bit capacity (32768 pages = 64 GiB)

// Side map layout (32-bit words).  The buffer must start zeroed.
enum : qrc_u32 {
    H_MAGIC = 0, H_STATUS = 1, H_MASK = 2, H_CHUNK_LOG2 = 3, H_NSM = 4, H_NSIDE0 = 5,
    H_NSIDE1 = 6, H_NPAGES = 7, H_BASE_LO = 8, H_BASE_HI = 9, H_BYTES_LO = 10, H_BYTES_HI = 11,
    H_VERIFY_N = 12, H_VERIFY_BAD = 13, H_LAT0 = 14, H_LAT1 = 15, H_INIT_TICKET = 16,
    H_RUN_TICKET = 17, H_ACC = 18, H_PAGE_WORDS_CAP = 19, H_MASK_MEASURED = 20,
    H_SM_C0 = 21, H_SM_C1 = 22, H_BIT_C0 = 23, H_BIT_C1 = 24, H_SMID_LAST = 25,
    H_QUEUE0 = 32, H_QUEUE1 = 64,                  // each on its own 128-byte line
    H_ERR = 96, H_ERR_ADDR_LO = 97, H_ERR_ADDR_HI = 98, H_WAIT_ERR = 99,
    H_COV_BYTES_LO = 100, H_COV_BYTES_HI = 101, H_COV_XOR_LO = 102, H_COV_XOR_HI = 103,
    H_ACC64 = 104,                                 // 8-byte aligned double accumulator (sums), 104..105
    H_XCHG_ERR = 106,                              // a peer's value never arrived (sticky until cleared)
    H_QUANT_TICKET = 107,                          // side-aware quantize pass: CTAs done
    H_EPOCH = 108,                                 // share-mark tag of the last launch with shares
    H_COPY_TICKET = 109,                           // side-aware copy: CTAs done
    H_FUSED_ARRIVE = 111,                          // fused quantize: CTAs past the amax phase
    H_FUSED_DONE = 112,                            // fused quantize: CTAs done (ticket)
    H_FUSED_ERR = 113,                             // fused quantize: a bounded wait gave up, or a share was missing
    H_FUSED_ACC = 114,                             // fused quantize: amax bits of this launch
    O_FUSED_SHARES = 120,                          // fused quantize: 8 words, shares read this launch
    H_FUSED_Q0 = 160, H_FUSED_Q1 = 192,            // fused quantize: phase-2 queues (own 128-byte lines)
    O_BITLAT = 128,                                // 21 raw latencies of the mask probes
    O_SM_SIDE = 256,                               // per SM: 0 unknown, else 1 + side + 2 * index within side
    O_SM_LAT = 512,                                // per SM raw anchor latency (cycles)
    O_PAGE_LAT = 1024,                             // first kDiagPages raw page latencies
    O_CLAIMS = 2048,                               // share marks (launch tags): side * 128 + index within side
    O_TIMELINE = 3072,                             // QRC_TIMELINE: 4 words per CTA, 256 CTAs
    O_PAGE_BITS = 4096,                            // one bit per 2 MiB page
};

enum : qrc_u32 {
    ST_OK = 0, ST_TOO_SMALL = 1, ST_NO_SM_SPLIT = 2, ST_NO_HASH = 3, ST_BAD_HASH = 4,
    ST_NO_CAL_SPLIT = 5, ST_VERIFY_FAILED = 6, ST_TOO_MANY_PAGES = 7, ST_UNALIGNED = 8,
};

enum : qrc_u32 { MODE_SIDE_AWARE = 0, MODE_IGNORE_PAGE_BITS = 1, MODE_WRONG_SIDE = 2, MODE_STREAM = 3 };
// Schedule bits, OR-ed into the mode: automatic by size, static shares, side
// queues, or static shares with a queued tail (see reduce_run).
enum : qrc_u32 { SCHED_AUTO = 0x00, SCHED_STATIC = 0x10, SCHED_QUEUE = 0x20, SCHED_BALANCED = 0x30,
                 SCHED_MASK = 0x30 };

QRC_DEV qrc_u32 smid() {
    qrc_u32 r;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
    return r;
}

QRC_DEV int parity64(qrc_u64 x) { return __popcll(x) & 1; }

// Programmatic dependent launch: wait for the preceding grid in the stream to
// complete (and its memory to be visible); allow the next grid to be scheduled
// while this one drains.  Both are no-ops unless the launch opted in.
QRC_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
QRC_DEV void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Cycles for kProbeIters dependent L2 atomics on `w`.  atomicCAS(w, v, v) with v
// the current value writes back the value it found, so memory never changes,
// and each CAS needs the previous result as its compare operand.  The first
// CAS (untimed) brings the line into L2.  The clock reads take the chain's
// value as an operand so they cannot move across it.
QRC_DEV qrc_u32 probe_latency(qrc_u32* w) {
    qrc_u32 v = atomicCAS(w, 0u, 0u);
    qrc_u64 t0, t1;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(t0) : "r"(v) : "memory");
    #pragma unroll 1
    for (int i = 0; i < kProbeIters; i++) v = atomicCAS(w, v, v);
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(t1) : "r"(v) : "memory");
    return (qrc_u32)(t1 - t0);
}

// 1-D two-means on n values (n small, one thread).  Returns false when there
// are fewer than two distinct values.  *lo/*hi are the cluster means.
QRC_DEV bool two_means(const qrc_u32* v, int n, float* lo, float* hi) {
    float mn = 3.4e38f, mx = 0.f;
    int cnt = 0;
    for (int i = 0; i < n; i++) {
        if (v[i] == 0) continue;
        mn = fminf(mn, (float)v[i]); mx = fmaxf(mx, (float)v[i]); cnt++;
    }
    if (cnt < 2 || !(mx > mn)) return false;
    float c0 = mn, c1 = mx;
    for (int it = 0; it < 32; it++) {
        const float t = 0.5f * (c0 + c1);
        float s0 = 0.f, s1 = 0.f; int n0 = 0, n1 = 0;
        for (int i = 0; i < n; i++) {
            if (v[i] == 0) continue;
            const float x = (float)v[i];
            if (x < t) { s0 += x; n0++; } else { s1 += x; n1++; }
        }
        if (n0 == 0 || n1 == 0) break;
        c0 = s0 / n0; c1 = s1 / n1;
    }
    *lo = c0; *hi = c1;
    return true;
}

// Separation required between near and far latency clusters (relative).
QRC_DEV bool separated(float lo, float hi) { return hi > lo * 1.04f + 8.0f; }

QRC_DEV qrc_u64 map_base(const qrc_u32* map) {
    return ((qrc_u64)map[H_BASE_HI] << 32) | map[H_BASE_LO];
}
QRC_DEV qrc_u64 map_bytes(const qrc_u32* map) {
    return ((qrc_u64)map[H_BYTES_HI] << 32) | map[H_BYTES_LO];
}

// ---------------------------------------------------------------------------
// Discovery
// ---------------------------------------------------------------------------

// Probe address of page p: its first word inside [a, end).
QRC_DEV qrc_u64 page_probe_addr(qrc_u64 a, qrc_u64 page_base, qrc_u64 p) {
    qrc_u64 x = page_base + p * kPage;
    if (x < a) x = (a + 3) & ~3ull;
    return x;
}

QRC_DEV void write_header_and_publish(qrc_u32* map, qrc_u32 status, qrc_u64 a, qrc_u64 bytes) {
    map[H_BASE_LO] = (qrc_u32)a; map[H_BASE_HI] = (qrc_u32)(a >> 32);
    map[H_BYTES_LO] = (qrc_u32)bytes; map[H_BYTES_HI] = (qrc_u32)(bytes >> 32);
    map[H_STATUS] = status;
    __threadfence();
    map[H_MAGIC] = kMagic;
    __threadfence();
}

QRC_DEV void discover(const void* A, qrc_u64 bytes, qrc_u32* map) {
    __shared__ int s_last;
    __shared__ qrc_u32 s_lat[64];
    __shared__ qrc_u32 s_cfg[8];   // 0 status, 1 mask, 2 lowbit, 3 thr, 4 near_is_0
    __shared__ int s_bad;

    // Probes are 4-byte atomics: only whole words inside [a, a + bytes) are touched.
    const qrc_u64 a = (qrc_u64)A, end = a + (bytes & ~3ull);
    const qrc_u64 anchor = (a + kPage - 1) & ~(kPage - 1);
    const bool big_enough = ((a & 3) == 0) && bytes >= kPage && anchor + kPage <= end;

    // ---- phase 1: every CTA times the anchor from its SM ----------------
    if (threadIdx.x == 0) {
        if (big_enough) {
            const qrc_u32 sm = smid();
            __nanosleep((sm & 7u) * 20000u);      // 8 waves, distinct words within a wave
            qrc_u32* w = (qrc_u32*)(anchor + 4ull * ((sm >> 3) & 31u));
            const qrc_u32 lat = probe_latency(w);
            if (sm < (qrc_u32)kMaxSm) map[O_SM_LAT + sm] = lat;
        }
        __threadfence();
        const qrc_u32 t = atomicInc(&map[H_INIT_TICKET], gridDim.x - 1);
        s_last = (t == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const qrc_u64 page_base = a & ~(kPage - 1);
    const qrc_u64 npages = (end - page_base + kPage - 1) / kPage;
    qrc_u32 cap_words = map[H_PAGE_WORDS_CAP];
    if (cap_words == 0) cap_words = kDefaultPageWords;

    if (!big_enough || W < 2) {
        if (threadIdx.x == 0) {
            map[H_NPAGES] = (qrc_u32)npages;
            write_header_and_publish(map, (a & 3) ? ST_UNALIGNED : ST_TOO_SMALL, a, bytes);
        }
        return;
    }

    // ---- SM classification (one thread) ----------------------------------
    // Other CTAs' latencies are read through L2 (ld.cg): they were written by
    // other SMs before their fenced ticket.
    __shared__ qrc_u32 s_smlat[kMaxSm];
    for (int i = threadIdx.x; i < kMaxSm; i += blockDim.x) s_smlat[i] = __ldcg(map + O_SM_LAT + i);
    __syncthreads();
    if (threadIdx.x == 0) {
        qrc_u32 st = ST_OK;
        float c0 = 0.f, c1 = 0.f;
        if (!two_means(s_smlat, kMaxSm, &c0, &c1) || !separated(c0, c1)) st = ST_NO_SM_SPLIT;
        const float thr = 0.5f * (c0 + c1);
        qrc_u32 n0 = 0, n1 = 0, nsm = 0;
        for (int i = 0; i < kMaxSm; i++) {
            const qrc_u32 l = s_smlat[i];
            if (l == 0) { map[O_SM_SIDE + i] = 0; continue; }
            nsm++;
            const qrc_u32 side = (st == ST_OK && (float)l >= thr) ? 1u : 0u;
            map[O_SM_SIDE + i] = 1u + side + 2u * (side ? n1 : n0);   // side and dense index within it
            if (side) n1++; else n0++;
        }
        map[H_NSM] = nsm; map[H_NSIDE0] = n0; map[H_NSIDE1] = n1;
        map[H_SM_C0] = (qrc_u32)c0; map[H_SM_C1] = (qrc_u32)c1;
        map[H_SMID_LAST] = smid();
        s_cfg[0] = st;
    }
    __syncthreads();

    // ---- mask discovery: 4 anchor probes + bits 4..20, one warp each ------
    for (int it = warp; it < 21; it += W) {
        if (lane == 0) {
            const qrc_u64 x = it < 4 ? anchor : (anchor ^ (1ull << it));
            s_lat[it] = probe_latency((qrc_u32*)x);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 0; i < 21; i++) map[O_BITLAT + i] = s_lat[i];
        qrc_u32 st = s_cfg[0], mask = 0, lowbit = 0;
        float c0 = 0.f, c1 = 0.f;
        if (st == ST_OK) {
            if (!two_means(s_lat, 21, &c0, &c1) || !separated(c0, c1)) {
                st = ST_NO_HASH;
            } else {
                const float thr = 0.5f * (c0 + c1);
                const bool anchor_hi = (float)(s_lat[0] + s_lat[1] + s_lat[2] + s_lat[3]) * 0.25f >= thr;
                bool anchors_agree = true;
                for (int i = 0; i < 4; i++) anchors_agree &= (((float)s_lat[i] >= thr) == anchor_hi);
                for (int b = 4; b <= 20; b++)
                    if ((((float)s_lat[b] >= thr) != anchor_hi)) mask |= 1u << b;
                if (!anchors_agree || mask == 0) st = ST_NO_HASH;
                else {
                    lowbit = __ffs(mask) - 1;
                    if (lowbit < 9) st = ST_BAD_HASH;   // chunk must hold >= one 512 B warp row
                }
            }
        }
        map[H_MASK_MEASURED] = mask;
        map[H_BIT_C0] = (qrc_u32)c0; map[H_BIT_C1] = (qrc_u32)c1;
        s_cfg[0] = st; s_cfg[1] = mask; s_cfg[2] = lowbit;
    }
    __syncthreads();
    qrc_u32 st = s_cfg[0];
    const qrc_u32 mask = s_cfg[1];
    const qrc_u64 partner = anchor ^ (1ull << s_cfg[2]);

    // ---- calibration wave: side-0 anchor vs side-1 partner -----------------
    if (st == ST_OK) {
        for (int it = warp; it < 2 * kCalProbes; it += W)
            if (lane == 0) s_lat[it] = probe_latency((qrc_u32*)((it & 1) ? partner : anchor));
        __syncthreads();
        if (threadIdx.x == 0) {
            float l0 = 0.f, l1 = 0.f;
            for (int i = 0; i < 2 * kCalProbes; i++) {
                if (i & 1) l1 += (float)s_lat[i]; else l0 += (float)s_lat[i];
            }
            l0 /= kCalProbes; l1 /= kCalProbes;
            map[H_LAT0] = (qrc_u32)l0; map[H_LAT1] = (qrc_u32)l1;
            if (!separated(fminf(l0, l1), fmaxf(l0, l1))) st = ST_NO_CAL_SPLIT;
            const qrc_u64 nwords = (npages + 31) / 32;
            if (nwords > cap_words) st = ST_TOO_MANY_PAGES;
            s_cfg[0] = st;
            s_cfg[3] = (qrc_u32)(0.5f * (l0 + l1));
            s_cfg[4] = l0 < l1;
        }
        __syncthreads();
        st = s_cfg[0];
    }
    const qrc_u32 thr = s_cfg[3];
    const bool near_is_0 = s_cfg[4] != 0;
    // side of an address from this SM's latency to it
    #define QRC_CLASSIFY(lat) ((((lat) < thr) == near_is_0) ? 0 : 1)

    // ---- page probes: warp k owns page-bit words k, k+W, ... --------------
    if (st == ST_OK) {
        const qrc_u64 nwords = (npages + 31) / 32;
        for (qrc_u64 wd = warp; wd < nwords; wd += W) {
            if (lane == 0) {
                qrc_u32 word = 0;
                for (int j = 0; j < 32; j++) {
                    const qrc_u64 p = wd * 32 + j;
                    if (p >= npages) break;
                    const qrc_u64 x = page_probe_addr(a, page_base, p);
                    const qrc_u32 lat = probe_latency((qrc_u32*)x);
                    if (p < (qrc_u64)kDiagPages) map[O_PAGE_LAT + p] = lat;
                    const qrc_u32 bit = (qrc_u32)QRC_CLASSIFY(lat) ^ (qrc_u32)parity64(x & mask);
                    word |= bit << j;
                }
                map[O_PAGE_BITS + wd] = word;
            }
        }
        if (threadIdx.x == 0) s_bad = 0;
        __syncthreads();

        // ---- verification: known anchors + pseudo-random words -----------
        const int nver = 2 * kVerifyCal + kVerifyRandom;
        for (int it = warp; it < nver; it += W) {
            if (lane == 0) {
                qrc_u64 x;
                if (it < kVerifyCal) x = anchor;
                else if (it < 2 * kVerifyCal) x = partner;
                else {
                    qrc_u64 h = (qrc_u64)(it + 1) * 0x9E3779B97F4A7C15ull;
                    h ^= h >> 29; h *= 0xBF58476D1CE4E5B9ull; h ^= h >> 32;
                    x = a + ((h % ((end - a) >> 2)) << 2);
                }
                const qrc_u64 p = (x - page_base) / kPage;
                const int pbit = (map[O_PAGE_BITS + (p >> 5)] >> (p & 31)) & 1;
                const int predicted = parity64(x & mask) ^ pbit;
                const int measured = QRC_CLASSIFY(probe_latency((qrc_u32*)x));
                if (predicted != measured) atomicAdd(&s_bad, 1);
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            map[H_VERIFY_N] = nver;
            map[H_VERIFY_BAD] = (qrc_u32)s_bad;
            if (s_bad * 8 > nver) st = ST_VERIFY_FAILED;
            s_cfg[0] = st;
        }
        __syncthreads();
        st = s_cfg[0];
    }
    #undef QRC_CLASSIFY

    if (threadIdx.x == 0) {
        map[H_MASK] = (st == ST_OK) ? mask : 0u;
        map[H_CHUNK_LOG2] = (st == ST_OK) ? s_cfg[2] : 12u;
        map[H_NPAGES] = (qrc_u32)npages;
        write_header_and_publish(map, st, a, bytes);
    }
}

// ---------------------------------------------------------------------------
// Reduction
// ---------------------------------------------------------------------------

// acc = maxNum(acc, |x|): IEEE-754 maxNum (a NaN operand loses), no FTZ.
QRC_DEV float absmax_step(float acc, float x) {
    float r;
    asm("{\n\t.reg .f32 t;\n\tabs.f32 t, %2;\n\tmax.f32 %0, %1, t;\n\t}" : "=f"(r) : "f"(acc), "f"(x));
    return r;
}

// acc = maxNum(acc, x) and minNum(acc, x).
QRC_DEV float max_step(float acc, float x) {
    float r;
    asm("max.f32 %0, %1, %2;" : "=f"(r) : "f"(acc), "f"(x));
    return r;
}
QRC_DEV float min_step(float acc, float x) {
    float r;
    asm("min.f32 %0, %1, %2;" : "=f"(r) : "f"(acc), "f"(x));
    return r;
}

// Order-preserving map of float bits to unsigned keys: key(a) < key(b) when
// a < b, and -0 below +0.
QRC_DEV qrc_u32 float_key(float f) {
    const qrc_u32 b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
QRC_DEV float key_float(qrc_u32 k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Same on two packed bf16 lanes (max.bf16x2 is maxNum as well).
QRC_DEV qrc_u32 absmax_step_bf16x2(qrc_u32 acc, qrc_u32 x) {
    qrc_u32 r;
    asm("{\n\t.reg .b32 t;\n\tabs.bf16x2 t, %2;\n\tmax.bf16x2 %0, %1, t;\n\t}" : "=r"(r) : "r"(acc), "r"(x));
    return r;
}

// Sixteen bytes of an operator's neutral element: fills the load slots of a
// partial batch, which are stepped like the others.
template <class Op>
QRC_DEV uint4 pad16() { return make_uint4(Op::kPad, Op::kPad, Op::kPad, Op::kPad); }

// Streaming 16-byte load (flavour chosen by QRC_LOAD_KIND).
template <int Kind>
QRC_DEV uint4 ld16(qrc_u64 addr) {
    uint4 v;
    if constexpr (Kind == 0) {
        asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(addr));
    } else if constexpr (Kind == 2) {
        asm volatile("{\n\t.reg .b64 pol;\n\tcreatepolicy.fractional.L2::evict_first.b64 pol, 1.0;\n\t"
                     "ld.global.nc.L1::no_allocate.L2::cache_hint.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4], pol;\n\t}"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(addr));
    } else if constexpr (Kind == 4) {
        asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(addr));
    } else {
        asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(addr));
    }
    return v;
}
QRC_DEV uint4 ld_stream16(qrc_u64 addr) { return ld16<QRC_LOAD_KIND>(addr); }

#if QRC_LOAD_KIND == 3
// 32-byte load (sm_100 256-bit global loads), as two uint4.
QRC_DEV void ld_stream32(qrc_u64 addr, uint4& a, uint4& b) {
    asm volatile("ld.global.nc.L1::no_allocate.L2::evict_first.L2::256B.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(a.x), "=r"(a.y), "=r"(a.z), "=r"(a.w), "=r"(b.x), "=r"(b.y), "=r"(b.z), "=r"(b.w)
                 : "l"(addr));
}
#endif

// Element operators.  Each gives its accumulator (Acc) and how a thread steps
// it over 16 loaded bytes or one element; to_red() turns a thread's
// accumulator into the value the block and the grid combine, through its
// Finish: FinishMaxU32 (unsigned max on 32-bit keys, neutral 0) or
// FinishSumF64 (double addition).  Idempotent operators may read an element
// twice; the others need every element exactly once.  publish() writes the
// launch's result (NaN when a bounded wait gave up).
struct FinishMaxU32;
struct FinishSumF64;
QRC_DEV float e4m3_scale_from_amax(float amax);
QRC_DEV float qrc_nan() { return __uint_as_float(0x7FFFFFFFu); }

// max |x| (maxNum: NaN elements lose; empty gives +0).  Result float.
struct OpAbsF32 {
    typedef float Acc;
    typedef FinishMaxU32 Finish;
    static constexpr int kElem = 4;
    static constexpr bool kIdempotent = true;
    static constexpr qrc_u32 kPad = 0u;   // element bits that leave the accumulator unchanged
    QRC_DEV Acc zero() { return 0.0f; }
    QRC_DEV Acc step16(Acc a, uint4 v) {
        a = absmax_step(a, __uint_as_float(v.x)); a = absmax_step(a, __uint_as_float(v.y));
        a = absmax_step(a, __uint_as_float(v.z)); a = absmax_step(a, __uint_as_float(v.w));
        return a;
    }
    QRC_DEV Acc step_elem(Acc a, qrc_u64 addr) { return absmax_step(a, *(const float*)addr); }
    QRC_DEV Acc merge(Acc a, Acc b) { return max_step(a, b); }
    QRC_DEV qrc_u32 to_red(Acc a) { return __float_as_uint(a); }   // a >= +0: bits order like values
    QRC_DEV void publish(void* out, float*, qrc_u32 r, bool err) {
        *(float*)out = err ? qrc_nan() : __uint_as_float(r);
    }
};

// max |x| of bf16 elements, two lanes per accumulator; publishes amax as a
// float and, when asked, the e4m3 scale 448 / amax.
struct OpAbsBF16 {
    typedef qrc_u32 Acc;   // two bf16 lanes
    typedef FinishMaxU32 Finish;
    static constexpr int kElem = 2;
    static constexpr bool kIdempotent = true;
    static constexpr qrc_u32 kPad = 0u;   // element bits that leave the accumulator unchanged
    QRC_DEV Acc zero() { return 0u; }
    QRC_DEV Acc step16(Acc a, uint4 v) {
        a = absmax_step_bf16x2(a, v.x); a = absmax_step_bf16x2(a, v.y);
        a = absmax_step_bf16x2(a, v.z); a = absmax_step_bf16x2(a, v.w);
        return a;
    }
    QRC_DEV Acc step_elem(Acc a, qrc_u64 addr) {
        return absmax_step_bf16x2(a, (qrc_u32)(*(const unsigned short*)addr));
    }
    QRC_DEV Acc merge(Acc a, Acc b) { return absmax_step_bf16x2(a, b); }
    QRC_DEV qrc_u32 to_red(Acc a) {
        const qrc_u32 lo = a << 16, hi = a & 0xFFFF0000u;   // bf16 -> f32 bits, both >= +0
        return lo > hi ? lo : hi;
    }
    QRC_DEV void publish(void* out, float* scale_out, qrc_u32 r, bool err) {
        const float amax = err ? qrc_nan() : __uint_as_float(r);
        *(float*)out = amax;
        if (scale_out) *scale_out = e4m3_scale_from_amax(amax);
    }
};

// max x (maxNum: NaN elements lose; empty or all-NaN gives -inf).
struct OpMaxF32 {
    typedef float Acc;
    typedef FinishMaxU32 Finish;
    static constexpr int kElem = 4;
    static constexpr bool kIdempotent = true;
    static constexpr qrc_u32 kPad = 0xFF800000u;   // element bits that leave the accumulator unchanged
    QRC_DEV Acc zero() { return __uint_as_float(0xFF800000u); }
    QRC_DEV Acc step16(Acc a, uint4 v) {
        a = max_step(a, __uint_as_float(v.x)); a = max_step(a, __uint_as_float(v.y));
        a = max_step(a, __uint_as_float(v.z)); a = max_step(a, __uint_as_float(v.w));
        return a;
    }
    QRC_DEV Acc step_elem(Acc a, qrc_u64 addr) { return max_step(a, *(const float*)addr); }
    QRC_DEV Acc merge(Acc a, Acc b) { return max_step(a, b); }
    QRC_DEV qrc_u32 to_red(Acc a) { return float_key(a); }      // key(-inf) > 0, the neutral
    QRC_DEV void publish(void* out, float*, qrc_u32 r, bool err) {
        *(float*)out = err ? qrc_nan() : (r < float_key(zero()) ? zero() : key_float(r));
    }
};

// min x (minNum: NaN elements lose; empty or all-NaN gives +inf).  The grid
// combines complemented keys with unsigned max.
struct OpMinF32 {
    typedef float Acc;
    typedef FinishMaxU32 Finish;
    static constexpr int kElem = 4;
    static constexpr bool kIdempotent = true;
    static constexpr qrc_u32 kPad = 0x7F800000u;   // element bits that leave the accumulator unchanged
    QRC_DEV Acc zero() { return __uint_as_float(0x7F800000u); }
    QRC_DEV Acc step16(Acc a, uint4 v) {
        a = min_step(a, __uint_as_float(v.x)); a = min_step(a, __uint_as_float(v.y));
        a = min_step(a, __uint_as_float(v.z)); a = min_step(a, __uint_as_float(v.w));
        return a;
    }
    QRC_DEV Acc step_elem(Acc a, qrc_u64 addr) { return min_step(a, *(const float*)addr); }
    QRC_DEV Acc merge(Acc a, Acc b) { return min_step(a, b); }
    QRC_DEV qrc_u32 to_red(Acc a) { return ~float_key(a); }
    QRC_DEV void publish(void* out, float*, qrc_u32 r, bool err) {
        *(float*)out = err ? qrc_nan() : (r < ~float_key(zero()) ? zero() : key_float(~r));
    }
};

// sum of x, accumulated in double (every element exactly once; NaN and
// infinities propagate as in IEEE addition).  Result double.
struct OpSumF32 {
    typedef double Acc;
    typedef FinishSumF64 Finish;
    static constexpr int kElem = 4;
    static constexpr bool kIdempotent = false;
    static constexpr qrc_u32 kPad = 0u;   // element bits that leave the accumulator unchanged
    QRC_DEV Acc zero() { return 0.0; }
    // Widening and adding in one asm block keeps the compiler from widening
    // all 32 loaded floats of a batch at once (which spilled).
    QRC_DEV Acc add(Acc a, qrc_u32 x) {
        double r;
        asm("{\n\t.reg .f64 t;\n\tcvt.f64.f32 t, %2;\n\tadd.rn.f64 %0, %1, t;\n\t}" : "=d"(r) : "d"(a), "r"(x));
        return r;
    }
    QRC_DEV Acc step16(Acc a, uint4 v) {
        a = add(a, v.x); a = add(a, v.y); a = add(a, v.z); a = add(a, v.w);
        return a;
    }
    QRC_DEV Acc step_elem(Acc a, qrc_u64 addr) { return add(a, *(const qrc_u32*)addr); }
    QRC_DEV Acc merge(Acc a, Acc b) { return a + b; }
    QRC_DEV double to_red(Acc a) { return a; }
    QRC_DEV void publish(void* out, float*, double r, bool err) {
        *(double*)out = err ? __longlong_as_double(0x7FF8000000000000ll) : r;
    }
};

// sum of x*x in double (fma per element).  Result double.
struct OpSumSqF32 {
    typedef double Acc;
    typedef FinishSumF64 Finish;
    static constexpr int kElem = 4;
    static constexpr bool kIdempotent = false;
    static constexpr qrc_u32 kPad = 0u;   // element bits that leave the accumulator unchanged
    QRC_DEV Acc zero() { return 0.0; }
    QRC_DEV Acc sq(Acc a, qrc_u32 x) {         // a + x*x, the square exact in double
        double r;
        asm("{\n\t.reg .f64 t;\n\tcvt.f64.f32 t, %2;\n\tfma.rn.f64 %0, t, t, %1;\n\t}" : "=d"(r) : "d"(a), "r"(x));
        return r;
    }
    QRC_DEV Acc step16(Acc a, uint4 v) {
        a = sq(a, v.x); a = sq(a, v.y); a = sq(a, v.z); a = sq(a, v.w);
        return a;
    }
    QRC_DEV Acc step_elem(Acc a, qrc_u64 addr) { return sq(a, *(const qrc_u32*)addr); }
    QRC_DEV Acc merge(Acc a, Acc b) { return a + b; }
    QRC_DEV double to_red(Acc a) { return a; }
    QRC_DEV void publish(void* out, float*, double r, bool err) {
        *(double*)out = err ? __longlong_as_double(0x7FF8000000000000ll) : r;
    }
};

#ifdef QRC_CHECKED
// Checked build: every access is tested against [lo, hi) before it is made;
// a bad one is recorded (first only) and skipped.  Coverage counters record the
// number of bytes read and an XOR of a hash of every 2-byte unit address read,
// which the host compares with the same quantities over the input range.
QRC_DEV qrc_u64 cov_hash(qrc_u64 x) {
    x ^= x >> 31; x *= 0x7FB5D329728EA185ull; x ^= x >> 27; x *= 0x81DADEF4BC2DD44Dull; x ^= x >> 33;
    return x;
}
struct CheckState { qrc_u64 lo, hi, bytes, xr; qrc_u32* map; };
QRC_DEV bool check_access(CheckState& cs, qrc_u64 addr, int size) {
    if (addr < cs.lo || addr + size > cs.hi || (addr & (size - 1))) {
        if (atomicCAS(&cs.map[H_ERR], 0u, 1u) == 0u) {
            cs.map[H_ERR_ADDR_LO] = (qrc_u32)addr; cs.map[H_ERR_ADDR_HI] = (qrc_u32)(addr >> 32);
        }
        return false;
    }
    cs.bytes += size;
    for (int i = 0; i < size; i += 2) cs.xr ^= cov_hash(addr + i);
    return true;
}
#define QRC_CS_PARAM , CheckState& cs
#define QRC_CS_ARG , cs
#define QRC_CHECK(addr, size) if (check_access(cs, (addr), (size)))
#else
#define QRC_CS_PARAM
#define QRC_CS_ARG
#define QRC_CHECK(addr, size)
#endif

// Element-wise pass over [x0, x1) by one warp (edges shorter than a pair).
template <class Op>
QRC_DEV typename Op::Acc edge_warp(typename Op::Acc acc, qrc_u64 x0, qrc_u64 x1, int lane QRC_CS_PARAM) {
    for (qrc_u64 x = x0 + (qrc_u64)Op::kElem * lane; x < x1; x += 32ull * Op::kElem) {
        QRC_CHECK(x, Op::kElem) acc = Op::step_elem(acc, x);
    }
    return acc;
}

// Reads one C-byte chunk (C >= 512) with a warp: lane l reads 16 bytes at
// l*16 + k*512 for k < C/512 (or, with 256-bit loads, 32 bytes at
// l*32 + k*1024); eight 16-byte loads' worth are kept in flight per lane.
template <class Op, int Kind = QRC_LOAD_KIND>
QRC_DEV typename Op::Acc chunk_warp(typename Op::Acc acc, qrc_u64 chunk, int n512, int lane QRC_CS_PARAM) {
#if QRC_LOAD_KIND == 3 && !defined(QRC_CHECKED)
    if (Kind == 3 && n512 >= 2) {
        const qrc_u64 base = chunk + 32ull * lane;
        const int n1k = n512 >> 1;
        for (int k = 0; k < n1k; k += 4) {
            uint4 v[8];
            #pragma unroll
            for (int u = 0; u < 4; u++) {
                v[2 * u] = v[2 * u + 1] = pad16<Op>();
                if (k + u < n1k) ld_stream32(base + 1024ull * (k + u), v[2 * u], v[2 * u + 1]);
            }
            #pragma unroll
            for (int u = 0; u < 8; u++) acc = Op::step16(acc, v[u]);
        }
        return acc;
    }
#endif
    const qrc_u64 base = chunk + 16ull * lane;
    for (int k = 0; k < n512; k += 8) {
        uint4 v[8];
        #pragma unroll
        for (int u = 0; u < 8; u++) {
            v[u] = pad16<Op>();
            const qrc_u64 x = base + 512ull * (k + u);
            if (k + u < n512) { QRC_CHECK(x, 16) v[u] = ld16<Kind>(x); }
        }
        #pragma unroll
        for (int u = 0; u < 8; u++) acc = Op::step16(acc, v[u]);
    }
    return acc;
}

// Reads up to 8 chunks with a warp, row k of every chunk before row k+1.
template <class Op>
QRC_DEV typename Op::Acc chunks_across(typename Op::Acc acc, const qrc_u64* ch, int m, int n512, int lane QRC_CS_PARAM) {
    for (int k = 0; k < n512; k++) {
        uint4 v[8];
        #pragma unroll
        for (int u = 0; u < 8; u++) {
            v[u] = pad16<Op>();
            const qrc_u64 x = ch[u] + 16ull * lane + 512ull * k;
            if (u < m) { QRC_CHECK(x, 16) v[u] = ld_stream16(x); }
        }
        #pragma unroll
        for (int u = 0; u < 8; u++) acc = Op::step16(acc, v[u]);
    }
    return acc;
}

// scale for an e4m3 per-tensor quantize: 448 / amax with IEEE round-to-nearest
// division; 1 when amax is 0 (empty / all-zero / all-NaN input) or infinite.
QRC_DEV float e4m3_scale_from_amax(float amax) {
    if (!(amax > 0.0f) || amax == __int_as_float(0x7F800000)) return 1.0f;
    return __fdiv_rn(448.0f, amax);
}

// Per-warp walk over the pairs of one side, for the pairs the static shares
// leave to the queues ([qbase, npairs)).  Built from the side map (or without
// one: mask 0, page bits 0), it hands each call the address of the next
// C-byte chunk this warp must read.  Work comes from the side's queue, a
// counter of positions: a warp adds its grab size and owns the positions
// between the old and new value; positions map to pairs through the
// interleave of pair_of().  For every pair the warp reads the half homed on
// its own side, so the two sides' queues together read every queued byte
// once whatever the map says.  Grabs are guided: QRC_MAX_GRAB pairs while
// plenty are left, shrinking to one pair as the queue empties.  The first
// request is issued by begin() without waiting (its reply is read on the
// first next()), and each later request while the current grab is read.
// All lanes call begin()/next() together (they broadcast lane 0's atomics).
// Geometry of one reduction: the pair range, the side map's mask and page
// bits, and this SM's side and index within it.  chunk_of() turns a pair into
// the address of its chunk homed on a given side.
struct ChunkMap {
    qrc_u64 lo, hi, C, mask, page_base, npairs;
    const qrc_u32* page_bits;
    int side, sm_index, use_page_bits, flip;
    bool aware;

    QRC_MEMBER void setup(qrc_u64 a, qrc_u64 end, const qrc_u32* map, qrc_u32 mode) {
        // Every header word is loaded unconditionally, so the loads go out
        // together (one round trip) before anything depends on them.
        const qrc_u32 sm = smid();
        const qrc_u32 h_magic = map[H_MAGIC], h_status = map[H_STATUS], h_mask = map[H_MASK];
        const qrc_u32 h_clog2 = map[H_CHUNK_LOG2];
        const qrc_u64 mb = map_base(map), mbytes = map_bytes(map);
        const qrc_u32 lab_raw = map[O_SM_SIDE + (sm & (qrc_u32)(kMaxSm - 1))];
        aware = h_magic == kMagic && h_status == ST_OK && a >= mb && end <= mb + mbytes;
        mask = aware ? h_mask : 0u;
        C = 1ull << (aware ? (int)h_clog2 : 12);
        page_base = mb & ~(kPage - 1);
        page_bits = map + O_PAGE_BITS;
        use_page_bits = aware && mode != MODE_IGNORE_PAGE_BITS;
        flip = mode == MODE_WRONG_SIDE;
        const qrc_u32 lab = (aware && sm < (qrc_u32)kMaxSm) ? lab_raw : 0u;
        side = lab ? (int)((lab - 1) & 1) : (int)(blockIdx.x & 1);
        sm_index = lab ? (int)((lab - 1) >> 1) : -1;
        const qrc_u64 PAIR = 2 * C;
        lo = (a + PAIR - 1) & ~(PAIR - 1);
        hi = end & ~(PAIR - 1);
        if (hi <= lo) { lo = end; hi = end; }
        npairs = (hi - lo) / PAIR;
    }
    // Address of the chunk of `pair` homed on side `s`.
    QRC_MEMBER qrc_u64 chunk_of(qrc_u64 pair, int s) const {
        const qrc_u64 pa = lo + pair * (2 * C);
        int pbit = 0;
        if (use_page_bits) {
            const qrc_u64 pg = (pa - page_base) >> 21;
            pbit = (page_bits[pg >> 5] >> (pg & 31)) & 1;
        }
        const int first_side = parity64(pa & mask) ^ pbit ^ flip;
        return pa + ((first_side != s) ? C : 0ull);
    }
};

struct SideWalk : ChunkMap {
    qrc_u64 qbase, nq, p, p1, nstart;
    qrc_u64 main_pairs, tail_stride;   // interleave over the nq queued pairs
    qrc_u32* queue;
    qrc_u32* other;
    qrc_u32 nsize, spread;
    bool pending, stealing;
    qrc_u32 stolen;                    // chunks read through the other side's queue

    QRC_MEMBER void setup(qrc_u64 a, qrc_u64 end, qrc_u32* map, qrc_u32 mode) {
        ChunkMap::setup(a, end, map, mode);
        queue = &map[side ? H_QUEUE1 : H_QUEUE0];
        other = &map[side ? H_QUEUE0 : H_QUEUE1];
        stealing = false;
        stolen = 0;
        spread = gridDim.x * (blockDim.x >> 5);     // ~2x the warps reading one side
        set_queued(0);
        p = p1 = nstart = 0;
        nsize = 0;
        pending = false;
    }
    // The queues cover pairs [first, npairs).
    QRC_MEMBER void set_queued(qrc_u64 first) {
        qbase = first;
        nq = npairs - first;
        const int block_log2 = kStrideLog2 ? kStrideLog2 + kGrabLog2 : 0;
        main_pairs = kStrideLog2 ? (nq >> block_log2) << block_log2 : 0;
        tail_stride = kStrideLog2 ? (nq - main_pairs) >> kGrabLog2 : 0;
    }
    // Grab size when `seen` queued positions of this side are taken.
    QRC_MEMBER qrc_u32 grab_size(qrc_u64 seen) const {
        if (stealing) return 1u;                 // the other side is in its tail
        const qrc_u64 left = nq > seen ? nq - seen : 0;
        const qrc_u64 s = left / spread;
        return s >= kMaxGrab ? kMaxGrab : (s < 1 ? 1u : (qrc_u32)s);
    }
    // Lane 0 requests the grab that follows [start, start + size).
    QRC_MEMBER void request(int lane, qrc_u64 start, qrc_u32 size) {
        if (lane == 0) {
            nsize = grab_size(start + size);
            nstart = atomicAdd(queue, nsize);
        }
        pending = true;
    }
    // Makes positions [st, st + sz) current (and requests the next grab);
    // an exhausted queue leaves nothing pending.
    QRC_MEMBER void adopt(int lane, qrc_u64 st, qrc_u32 sz) {
        if (st >= nq) { p = p1 = 0; pending = false; return; }
        p = st;
        p1 = st + sz < nq ? st + sz : nq;
        request(lane, st, sz);
    }
    // Takes over a first request issued before the walk was built: lane 0's
    // `st` is the counter value returned for a grab of `sz` positions.
    QRC_MEMBER void begin_with(qrc_u64 st, qrc_u32 sz) {
        p = p1 = 0;
        nstart = st;
        nsize = sz;
        pending = nq > 0;
    }
    // First request; does not wait for the reply.
    QRC_MEMBER void begin(int lane) {
        p = p1 = 0;
        pending = false;
        if (nq == 0) return;
        if (lane == 0) {
            nsize = grab_size(0);
            nstart = atomicAdd(queue, nsize);
        }
        pending = true;
    }
    // Pair index (within the queued region) of queue position c: a bijection
    // of [0, nq).  Inside a block of 2^(stride+grab) positions, position r
    // goes to (r mod grab) * 2^stride + r / grab; the last, partial block uses
    // the stride that fits it; positions past that map to themselves.
    QRC_MEMBER qrc_u64 pair_of(qrc_u64 c) const {
        if (kStrideLog2 == 0) return c;
        const qrc_u64 G1 = (1ull << kGrabLog2) - 1;
        if (c < main_pairs) {
            const int block_log2 = kStrideLog2 + kGrabLog2;
            const qrc_u64 r = c & ((1ull << block_log2) - 1);
            return (c - r) + ((r & G1) << kStrideLog2) + (r >> kGrabLog2);
        }
        const qrc_u64 r = c - main_pairs;
        if (r < (tail_stride << kGrabLog2)) return main_pairs + (r & G1) * tail_stride + (r >> kGrabLog2);
        return c;
    }
    QRC_MEMBER qrc_u64 next(int lane) {
        while (p >= p1) {
            if (!pending) {
#if QRC_STEAL
                if (stealing || nq == 0) return 0;
                // Own side done: help the other side finish (its halves are
                // homed on the other die, so these reads cross it).
                stealing = true;
                side ^= 1;
                queue = other;
                begin(lane);
                continue;
#else
                return 0;
#endif
            }
            const qrc_u64 st = __shfl_sync(0xFFFFFFFFu, nstart, 0);
            const qrc_u32 sz = __shfl_sync(0xFFFFFFFFu, nsize, 0);
            adopt(lane, st, sz);
        }
        const qrc_u64 pair = qbase + pair_of(p);
        p++;
        stolen += stealing ? 1u : 0u;
        return chunk_of(pair, side);
    }
};

// ---- bulk-copy staging (cp.async.bulk global -> shared, mbarrier completion) ----

QRC_DEV void mbar_init(qrc_u32 bar, qrc_u32 count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}
QRC_DEV void mbar_arrive_expect_tx(qrc_u32 bar, qrc_u32 bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}
QRC_DEV bool mbar_try_wait(qrc_u32 bar, qrc_u32 parity) {
    qrc_u32 ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// Waits for the phase with the given parity to complete; gives up after
// kWaitCycles SM clocks and returns false.
constexpr long long kWaitCycles = 1ll << 31;   // about one second
QRC_DEV bool mbar_wait_bounded(qrc_u32 bar, qrc_u32 parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kWaitCycles) return false;
    return true;
}
QRC_DEV void bulk_g2s(qrc_u32 dst, qrc_u64 src, qrc_u32 bytes, qrc_u32 bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
QRC_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
QRC_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

constexpr qrc_u32 kSlotBytes = 4096;                  // one staging slot
constexpr qrc_u32 kSlotStride = kSlotBytes + 8;       // slot + its mbarrier, for sizing
QRC_DEV int bulk_slots_per_warp(qrc_u32 dyn_smem_bytes, int warps) {
    const int s = (int)(dyn_smem_bytes / ((qrc_u32)warps * kSlotStride));
    return s > 16 ? 16 : s;
}
QRC_DEV qrc_u32 dynamic_smem_size() {
    qrc_u32 r;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(r));
    return r;
}

// Bulk variant of the side-aware walk: each warp owns S slots of 4 KiB in
// dynamic shared memory with one mbarrier each; lane 0 keeps every slot
// filled with the warp's next chunk through cp.async.bulk (one 1-D copy per
// slot, no multicast), all lanes wait for the slot, reduce it from shared
// memory and hand it back.  Up to warps * S * 4 KiB per SM are in flight
// without using registers.  Waits are bounded: on a timeout the warp records
// H_WAIT_ERR, drains its own copies (again bounded) and stops; the launch then
// publishes NaN instead of a maximum.
template <class Op>
QRC_DEV typename Op::Acc bulk_walk(typename Op::Acc acc, SideWalk& w, int S, qrc_u32* map, int lane, int warp) {
    extern __shared__ __align__(128) unsigned char qrc_dsmem[];
    const int W = blockDim.x >> 5;
    const qrc_u32 U = w.C < kSlotBytes ? (qrc_u32)w.C : kSlotBytes;   // bytes per copy
    const int per_chunk = (int)(w.C / U);
    const qrc_u32 slots = (qrc_u32)__cvta_generic_to_shared(qrc_dsmem) + (qrc_u32)(warp * S) * kSlotBytes;
    const qrc_u32 bars = (qrc_u32)__cvta_generic_to_shared(qrc_dsmem) + (qrc_u32)(W * S) * kSlotBytes + (qrc_u32)(warp * S) * 8u;
    if (lane == 0) {
        for (int s = 0; s < S; s++) mbar_init(bars + 8u * s, 1);
        fence_mbar_init();
        fence_proxy_async_smem();
    }
    __syncwarp();

    qrc_u64 chunk = 0;
    int k = per_chunk;
    auto next_unit = [&]() -> qrc_u64 {
        if (k == per_chunk) { chunk = w.next(lane); k = 0; }
        if (!chunk) return 0;
        return chunk + (qrc_u64)(k++) * U;
    };
    w.begin(lane);
    qrc_u32 valid = 0, parity = 0;
    for (int s = 0; s < S; s++) {
        const qrc_u64 src = next_unit();
        if (!src) break;
        valid |= 1u << s;
        if (lane == 0) { mbar_arrive_expect_tx(bars + 8u * s, U); bulk_g2s(slots + s * kSlotBytes, src, U, bars + 8u * s); }
    }
    int s = 0;
    bool failed = false;
    const int n512 = (int)(U >> 9);
    while (valid) {
        if (valid & (1u << s)) {
            if (!mbar_wait_bounded(bars + 8u * s, (parity >> s) & 1u)) { failed = true; break; }
            parity ^= 1u << s;
            const unsigned char* sp = qrc_dsmem + (size_t)(warp * S + s) * kSlotBytes + 16 * lane;
            if (n512 == 8) {
                uint4 v[8];
                #pragma unroll
                for (int u = 0; u < 8; u++) v[u] = *(const uint4*)(sp + 512 * u);
                #pragma unroll
                for (int u = 0; u < 8; u++) acc = Op::step16(acc, v[u]);
            } else {
                for (int u = 0; u < n512; u++) acc = Op::step16(acc, *(const uint4*)(sp + 512 * u));
            }
            __syncwarp();
            const qrc_u64 src = next_unit();
            if (src) {
                if (lane == 0) {
                    fence_proxy_async_smem();       // our generic reads of the slot before the async refill
                    mbar_arrive_expect_tx(bars + 8u * s, U);
                    bulk_g2s(slots + s * kSlotBytes, src, U, bars + 8u * s);
                }
            } else {
                valid &= ~(1u << s);
            }
        }
        s = (s + 1 == S) ? 0 : s + 1;
    }
    if (failed) {
        if (lane == 0) atomicOr(&map[H_WAIT_ERR], 1u);
        for (int t = 0; t < S; t++)                     // drain this warp's copies, bounded
            if (valid & (1u << t)) mbar_wait_bounded(bars + 8u * t, (parity >> t) & 1u);
    }
    return acc;
}

// Sum of the checked build's per-thread coverage counters into the map.
#ifdef QRC_CHECKED
QRC_DEV void cov_flush(CheckState& cs, int lane, qrc_u32* map) {
    qrc_u64 b = cs.bytes, x = cs.xr;
    for (int o = 16; o > 0; o >>= 1) {
        b += __shfl_xor_sync(0xFFFFFFFFu, b, o);
        x ^= __shfl_xor_sync(0xFFFFFFFFu, x, o);
    }
    if (lane == 0) {
        atomicAdd((unsigned long long*)&map[H_COV_BYTES_LO], b);
        atomicXor((unsigned long long*)&map[H_COV_XOR_LO], x);
    }
    cs.bytes = 0; cs.xr = 0;
}
#endif

// Maximum of `bits` over the block, returned to every thread.
QRC_DEV qrc_u32 block_max(qrc_u32 bits) {
    __shared__ qrc_u32 s_w[32];
    __shared__ qrc_u32 s_res;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    bits = __reduce_max_sync(0xFFFFFFFFu, bits);
    if (lane == 0) s_w[warp] = bits;
    __syncthreads();
    if (warp == 0) {
        qrc_u32 v = lane < W ? s_w[lane] : 0u;
        v = __reduce_max_sync(0xFFFFFFFFu, v);
        if (lane == 0) s_res = v;
    }
    __syncthreads();
    return s_res;
}

// Sum of `v` over the block, returned to every thread.
QRC_DEV double block_sum_f64(double v) {
    __shared__ double s_wd[32];
    __shared__ double s_resd;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    if (lane == 0) s_wd[warp] = v;
    __syncthreads();
    if (warp == 0) {
        double x = lane < W ? s_wd[lane] : 0.0;
        for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xFFFFFFFFu, x, o);
        if (lane == 0) s_resd = x;
    }
    __syncthreads();
    return s_resd;
}

// How blocks and the grid combine an operator's values (see the element
// operators): block(), a fire-and-forget global reduction into the map, and
// the last CTA's take-and-reset of the global accumulator.
// Cross-GPU combine of the launch's value (see XchgArgs): each rank stores
// (epoch, value) in its slot of every rank's slot array over NVLink, then
// waits, bounded, until its own array holds this epoch from every rank.
struct XchgArgs {
    qrc_u64* local;                  // this rank's slots: 2 (epoch parity) x world
    qrc_u64* const* peers;           // every rank's slot array, peers[rank] == local
    qrc_u32 rank, world, epoch;      // world <= 1: no exchange
};
constexpr long long kXchgWaitCycles = 1ll << 32;   // ~2 s at 2 GHz

// Warp 0 of the last CTA, every lane: max of `r` over all ranks; false on
// timeout.  Lane p (and p + 32) stores this rank's (epoch, value) word into
// rank p's slot array and polls this rank's slot for rank p, so the N stores
// and the N polls go out in parallel; the warp then takes the maximum.
QRC_DEV bool xchg_max_u32(const XchgArgs& x, qrc_u32& r, int lane) {
    const qrc_u32 par = x.epoch & 1u;
    const qrc_u64 word = ((qrc_u64)x.epoch << 32) | r;
    for (qrc_u32 p = (qrc_u32)lane; p < x.world; p += 32) {
        qrc_u64* dst = x.peers[p] + par * x.world + x.rank;
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" :: "l"(dst), "l"(word) : "memory");
    }
    const long long t0 = clock64();
    qrc_u32 m = r;
    bool ok = true;
    for (qrc_u32 q = (qrc_u32)lane; q < x.world && ok; q += 32) {
        qrc_u64 v;
        for (;;) {
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(x.local + par * x.world + q) : "memory");
            if ((qrc_u32)(v >> 32) == x.epoch) break;
            if (clock64() - t0 > kXchgWaitCycles) { ok = false; break; }
            __nanosleep(64);
        }
        if (ok) {
            const qrc_u32 val = (qrc_u32)v;
            m = m > val ? m : val;
        }
    }
    r = __reduce_max_sync(0xFFFFFFFFu, m);
    return __all_sync(0xFFFFFFFFu, ok);
}

struct FinishMaxU32 {
    typedef qrc_u32 Red;
    QRC_DEV bool exchange(const XchgArgs& x, Red& r, int lane) { return xchg_max_u32(x, r, lane); }
    QRC_DEV Red neutral() { return 0u; }
    QRC_DEV Red block(Red v) { return block_max(v); }
    QRC_DEV Red combine(Red a, Red b) { return a > b ? a : b; }
    QRC_DEV void red(qrc_u32* map, Red v) {
        asm volatile("red.relaxed.gpu.global.max.u32 [%0], %1;" :: "l"(&map[H_ACC]), "r"(v) : "memory");
    }
    QRC_DEV Red take(qrc_u32* map) { return atomicExch(&map[H_ACC], 0u); }
};
struct FinishSumF64 {
    typedef double Red;
    QRC_DEV bool exchange(const XchgArgs&, Red&, int) { return false; }   // not offered for sums
    QRC_DEV Red neutral() { return 0.0; }
    QRC_DEV Red block(Red v) { return block_sum_f64(v); }
    QRC_DEV Red combine(Red a, Red b) { return a + b; }
    QRC_DEV void red(qrc_u32* map, Red v) {
        asm volatile("red.relaxed.gpu.global.add.f64 [%0], %1;" :: "l"(&map[H_ACC64]), "d"(v) : "memory");
    }
    QRC_DEV Red take(qrc_u32* map) {
        return __longlong_as_double((long long)atomicExch((unsigned long long*)&map[H_ACC64], 0ull));
    }
};

// Static shares (see reduce_run).  All K_s SMs of side s take part; the two
// sides are not paired, each covers its own chunk of every pair.
// A 256-thread group reads the side-s chunks of 8 consecutive pairs at once:
// thread t loads bytes 16t..16t+15 of each of the 8 chunks (eight 16-byte
// loads in flight, all addresses computed on the spot).  Block b of 8 pairs
// belongs to group b mod (K_s * G) of side s, G = groups per CTA, and group g
// of the CTA on the SM with index k is group
//   * g * K_s + k when the shares are the whole input and R <=
//     QRC_SM_FIRST_MAX_PAIRS: consecutive blocks go to
//     different SMs, so a small input spreads over as many SMs as it has
//     blocks (4 MB: 64 SMs of a side with 32 KiB each, not 16 with 128 KiB)
//     and the SMs' totals differ by at most one block;
//   * k * G + g above that, so each SM steps through 8*G adjacent pairs, which
//     reads faster from DRAM when every SM has many blocks.
// Either way the K_s SMs of a side sweep one window of K_s * G blocks.
// Requires 4 KiB chunks (one 16-byte load per thread covers a chunk).
struct Shares {
    qrc_u64 R;          // pairs [0, R) are shared out statically
    qrc_u32 K0, K1;     // SMs per side
    bool on;
    bool sm_first;      // group of (k, g) is g * K_s + k, else k * G + g
    QRC_MEMBER qrc_u32 sms(int s) const { return s ? K1 : K0; }
    // First block of group g of SM k of side s.
    QRC_MEMBER qrc_u64 first_block(int s, int k, int g) const {
        return sm_first ? (qrc_u64)g * sms(s) + k : (qrc_u64)k * (blockDim.x >> 8) + g;
    }
};

// Page-bit word of 8-pair block b when the share fast path (64 KiB aligned
// body) reads it, else 0.  Page bits are written only by discovery, so this
// load may go out before the wait on the previous grid.
QRC_DEV qrc_u32 block_page_word(const ChunkMap& w, const Shares& sh, qrc_u64 b) {
    if (!w.use_page_bits || (w.lo & 0xFFFFull) != 0 || (b + 1) * 8 > sh.R) return 0u;
    const qrc_u64 pg = (w.lo + (b << 16) - w.page_base) >> 21;
    return w.page_bits[pg >> 5];
}
// `word0` is page-bit word 0, loaded with the map header: a share whose first
// block lies in the first 64 MiB of the mapped buffer needs no second load.
// The share is that of SM k of side s.
QRC_DEV qrc_u32 share_first_page_word(const ChunkMap& w, const Shares& sh, int s, int k, qrc_u32 word0) {
    const qrc_u64 b = sh.first_block(s, k, threadIdx.x >> 8);
    if (!w.use_page_bits || (w.lo & 0xFFFFull) != 0 || (b + 1) * 8 > sh.R) return 0u;
    const qrc_u64 pg = (w.lo + (b << 16) - w.page_base) >> 21;
    return (pg >> 5) == 0 ? word0 : w.page_bits[pg >> 5];
}

// `pw` is share_first_page_word(w, sh, s, k).
template <class Op, int Kind = QRC_LOAD_KIND>
QRC_DEV typename Op::Acc read_share(typename Op::Acc acc, const ChunkMap& w, const Shares& sh, int s, int k,
                                    qrc_u32 pw QRC_CS_PARAM) {
    const int G = blockDim.x >> 8, g = threadIdx.x >> 8, t = threadIdx.x & 255;
    const qrc_u64 groups = (qrc_u64)sh.sms(s) * G, npairs = sh.R;
    qrc_u64 b = sh.first_block(s, k, g);
    if ((w.lo & 0xFFFFull) == 0) {
        // Fast path: a block is 64 KiB aligned, so its 8 pairs share one page
        // bit, and pair j's masked-address parity is the block's XOR bit j of
        // `pat` (address bits 13-15 are j).  One popc per block; the page-bit
        // word of the next block is loaded with this block's data.
        qrc_u32 pat = 0;
        #pragma unroll
        for (int j = 0; j < 8; j++) pat |= (qrc_u32)parity64(((qrc_u64)j << 13) & w.mask) << j;
        for (; (b + 1) * 8 <= npairs; b += groups) {
            const qrc_u64 base = w.lo + (b << 16);
            const int pbit = (int)(pw >> (((base - w.page_base) >> 21) & 31)) & 1;
            pw = block_page_word(w, sh, b + groups);
            // chunk j is the second half when its first half is homed off side s
            const qrc_u32 second = (qrc_u32)(parity64(base & w.mask) ^ pbit ^ w.flip ^ s) ? ~pat : pat;
            const qrc_u64 row = base + 16ull * t;
            uint4 v[8];
            #pragma unroll
            for (int j = 0; j < 8; j++) {
                const qrc_u64 x = row + ((qrc_u64)j << 13) + ((qrc_u64)((second >> j) & 1u) << 12);
                QRC_CHECK(x, 16) v[j] = ld16<Kind>(x);
            }
            #pragma unroll
            for (int j = 0; j < 8; j++) acc = Op::step16(acc, v[j]);
        }
    }
    for (; b * 8 < npairs; b += groups) {
        uint4 v[8];
        #pragma unroll
        for (int j = 0; j < 8; j++) {
            v[j] = pad16<Op>();
            const qrc_u64 pair = b * 8 + j;
            if (pair < npairs) {
                const qrc_u64 x = w.chunk_of(pair, s) + 16ull * t;
                QRC_CHECK(x, 16) v[j] = ld16<Kind>(x);
            }
        }
        #pragma unroll
        for (int j = 0; j < 8; j++) acc = Op::step16(acc, v[j]);
    }
    return acc;
}

QRC_DEV void group_bar(int g) {
    asm volatile("bar.sync %0, 256;" :: "r"(1 + g) : "memory");
}

// Tail of the balanced schedule: pairs [R, npairs) in 8-pair blocks, taken one
// block per claim from the side's queue by each 256-thread group (the group's
// first thread claims, a named barrier hands the claim to the group).  The
// next claim is in flight while the current block is read.  When its own
// queue is empty, a group helps the other side (far reads).  `first` is the
// group leader's first claim, issued before the static share was read.
template <class Op, int Kind = QRC_LOAD_KIND>
QRC_DEV typename Op::Acc read_tail(typename Op::Acc acc, const ChunkMap& w, qrc_u64 R, qrc_u32* map, int s,
                                   qrc_u32 first QRC_CS_PARAM) {
    __shared__ qrc_u32 s_claim[2][4];
    const int g = threadIdx.x >> 8, t = threadIdx.x & 255;
    const bool leader = t == 0;
    const qrc_u64 nb = (w.npairs - R + 7) >> 3;
    const bool fast = ((w.lo + (R << 13)) & 0xFFFFull) == 0;
    qrc_u32 pat = 0;
    #pragma unroll
    for (int j = 0; j < 8; j++) pat |= (qrc_u32)parity64(((qrc_u64)j << 13) & w.mask) << j;
    qrc_u32* queue = &map[s ? H_QUEUE1 : H_QUEUE0];
    bool stealing = false;
    int par = 0;
    if (leader) s_claim[0][g] = first;
    group_bar(g);
    qrc_u32 cur = s_claim[0][g];
    for (;;) {
        qrc_u32 nxt = 0;
        if (cur >= nb) {
            if (stealing || !QRC_STEAL) break;
            stealing = true;
            s ^= 1;
            queue = &map[s ? H_QUEUE1 : H_QUEUE0];
            if (leader) nxt = atomicAdd(queue, 1u);
        } else {
            if (leader) nxt = atomicAdd(queue, 1u);
            const qrc_u64 p0 = R + ((qrc_u64)cur << 3);
            uint4 v[8];
            if (fast && p0 + 8 <= w.npairs) {
                const qrc_u64 base = w.lo + (p0 << 13);
                int pbit = 0;
                if (w.use_page_bits) {
                    const qrc_u64 pg = (base - w.page_base) >> 21;
                    pbit = (int)(w.page_bits[pg >> 5] >> (pg & 31)) & 1;
                }
                const qrc_u32 second = (qrc_u32)(parity64(base & w.mask) ^ pbit ^ w.flip ^ s) ? ~pat : pat;
                const qrc_u64 row = base + 16ull * t;
                #pragma unroll
                for (int j = 0; j < 8; j++) {
                    const qrc_u64 x = row + ((qrc_u64)j << 13) + ((qrc_u64)((second >> j) & 1u) << 12);
                    QRC_CHECK(x, 16) v[j] = ld16<Kind>(x);
                }
            } else {
                #pragma unroll
                for (int j = 0; j < 8; j++) {
                    v[j] = pad16<Op>();
                    const qrc_u64 pair = p0 + j;
                    if (pair < w.npairs) {
                        const qrc_u64 x = w.chunk_of(pair, s) + 16ull * t;
                        QRC_CHECK(x, 16) v[j] = ld16<Kind>(x);
                    }
                }
            }
            #pragma unroll
            for (int j = 0; j < 8; j++) acc = Op::step16(acc, v[j]);
        }
        // A slot is rewritten two barriers after it was read.
        par ^= 1;
        if (leader) s_claim[par][g] = nxt;
        group_bar(g);
        cur = s_claim[par][g];
    }
    return acc;
}

// The reduction over n elements at A (element type given by Op).
//
// Side-aware path (modes 0-2), register loads:
//   * Static shares: discovery gave every SM its side s and a dense index k
//     among the K_s SMs of that side.  The CTA on SM (s, k) reads the side-s
//     chunks of its share of pairs [0, R) (see read_share).  No atomics.  The
//     CTA marks its share with a plain store.  R is every pair (static
//     schedule), or 5/8 of them, 1/8 above 1 GiB (balanced schedule,
//     QRC_STATIC_EIGHTHS, QRC_STATIC_EIGHTHS_LARGE).
//   * Balanced schedule: the pairs past R go in 8-pair blocks through the
//     side queues, one block per claim by each 256-thread group (read_tail),
//     so SMs that run slower than the static split assumes (the spread across
//     SMs of one side reaches ~7 % on B200) are absorbed, and a side that
//     runs out helps the other.  The first claim is issued before the share
//     is read.
//   * Queue schedule: no shares; warps take one-pair grabs (SideWalk).
//   * A maximum does not change when an element is read twice, so two CTAs on
//     one SM only cost time.  A share nobody marked (an SM that got no CTA,
//     e.g. a grid smaller than the GPU) is read by the last CTA after the
//     ticket, before it publishes: every element is still read.
//   * Shares are used when one CTA fills an SM (1024 threads, or a block with
//     the bulk ring's shared memory), the block is a multiple of 256 threads,
//     chunks are 4 KiB and there is a valid side map; otherwise every pair
//     goes through the side queues (SideWalk).
// Bulk pipeline (dynamic shared memory for >= 2 slots per warp): queues only.
// Mode 3: side-agnostic grid-stride stream.
template <class Op>
QRC_DEV void reduce_run(const void* A, qrc_u64 n, qrc_u32* map, void* out, float* scale_out, qrc_u32 mode,
                        XchgArgs xa = XchgArgs{nullptr, nullptr, 0u, 0u, 0u}) {
    typedef typename Op::Finish Fin;
    const qrc_u32 sched = mode & SCHED_MASK;
    mode &= ~SCHED_MASK;
    const qrc_u64 a = (qrc_u64)A, bytes = n * (qrc_u64)Op::kElem, end = a + bytes;
    // Inputs that can stay in L2 between launches are read with plain loads,
    // which kept them resident where the non-coherent path did not.
    const bool plain = bytes <= (qrc_u64)QRC_PLAIN_MAX_BYTES;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    typename Op::Acc acc = Op::zero();
#ifdef QRC_CHECKED
    CheckState cs{a, end, 0ull, 0ull, map};
#endif
    qrc_u64 lo, hi;   // body [lo, hi); edges [a, lo) and [hi, end)
    Shares sh;
    __shared__ qrc_u32 s_tag;                        // this launch's share-mark tag (share path)
    __shared__ qrc_u32 s_mark;                       // map word of this CTA's share mark, 0 if none
    sh.on = false;
    sh.sm_first = false;
    sh.K0 = sh.K1 = 0;

    if (mode == MODE_STREAM) {
        // Side-agnostic grid-stride stream over the 16-byte aligned body.
        griddep_wait();
        lo = (a + 15) & ~15ull; hi = end & ~15ull;
        if (hi <= lo) { lo = end; hi = end; }
        const qrc_u64 nv = (hi - lo) / 16;
        const qrc_u64 tid = (qrc_u64)blockIdx.x * blockDim.x + threadIdx.x;
        const qrc_u64 stride = (qrc_u64)gridDim.x * blockDim.x;
        for (qrc_u64 i = tid; i < nv; i += 8 * stride) {
            uint4 v[8];
            #pragma unroll
            for (int u = 0; u < 8; u++) {
                v[u] = pad16<Op>();
                const qrc_u64 j = i + u * stride;
                if (j < nv) { QRC_CHECK(lo + 16 * j, 16) v[u] = ld_stream16(lo + 16 * j); }
            }
            #pragma unroll
            for (int u = 0; u < 8; u++) acc = Op::step16(acc, v[u]);
        }
        griddep_launch_dependents();
    } else {
        ChunkMap cm;
        cm.setup(a, end, map, mode);      // reads only the map header, which reductions never write
        // These go out with the header loads (one round trip for all): nothing
        // that decides whether they are needed may wait for that reply.
        const qrc_u32 word0 = map[O_PAGE_BITS];
        const qrc_u32 k0 = map[H_NSIDE0], k1 = map[H_NSIDE1];
        lo = cm.lo; hi = cm.hi;
        const int S = bulk_slots_per_warp(dynamic_smem_size(), W);
        sh.on = QRC_SHARES && cm.aware && S < 2 && cm.C == 4096 && (blockDim.x & 255) == 0 &&
                blockDim.x <= 1024 && (blockDim.x == 1024 || dynamic_smem_size() > 116u * 1024u) &&
                sched != SCHED_QUEUE;
        if (sh.on) {
            sh.K0 = k0;
            sh.K1 = k1;
            sh.on = k0 > 0 && k1 > 0 && k0 <= 128 && k1 <= 128;
            const bool tail = sched == SCHED_BALANCED ||
                              (sched == SCHED_AUTO && cm.npairs > (qrc_u64)QRC_STATIC_MAX_PAIRS);
            const qrc_u64 eighths = cm.npairs > (qrc_u64)QRC_LARGE_PAIRS ? QRC_STATIC_EIGHTHS_LARGE : QRC_STATIC_EIGHTHS;
            sh.R = tail ? (cm.npairs * eighths / 8) & ~7ull : cm.npairs;   // whole 8-pair blocks
            sh.sm_first = !tail && sh.R <= (qrc_u64)QRC_SM_FIRST_MAX_PAIRS;
        }
        const int own_k = cm.sm_index;
        const bool own_share = sh.on && own_k >= 0 && (qrc_u32)own_k < sh.sms(cm.side);
        const qrc_u32 pw0 = own_share ? share_first_page_word(cm, sh, cm.side, own_k, word0) : 0u;
        griddep_wait();                   // the scratch of the previous launch is reset
#if QRC_TIMELINE
        qrc_u64 t_start;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_start));
        qrc_u32 stolen = 0;
        if (blockIdx.x == 0 && threadIdx.x == 0)       // previous launch's finish, before this one overwrites it
            map[O_TIMELINE + 1022] = __ldcg(&map[O_TIMELINE + 1023]);
#endif
        if (sh.on) {
            // The tail's first claim goes out now; only its reply stays live
            // while the share is read.  A share's mark holds the tag of the
            // launch that read it (last launch's tag + 1), so marks need no
            // reset between launches.
            const bool tail = cm.npairs > sh.R;
            qrc_u32 first = 0;
            if (tail && (threadIdx.x & 255) == 0) first = atomicAdd(&map[cm.side ? H_QUEUE1 : H_QUEUE0], 1u);
            // The last warp fetches the tag (it alone waits for the reply);
            // the finish, after its barriers, writes the mark.
            if (threadIdx.x == blockDim.x - 32) s_tag = __ldcg(&map[H_EPOCH]) + 1u;
            if (threadIdx.x == 0) s_mark = own_share ? O_CLAIMS + 128 * cm.side + own_k : 0u;
            if (own_share) {
                if constexpr (Op::kIdempotent) {
                    // two CTAs on one SM both read the share: harmless
                    acc = plain ? read_share<Op, 0>(acc, cm, sh, cm.side, own_k, pw0 QRC_CS_ARG)
                                : read_share<Op>(acc, cm, sh, cm.side, own_k, pw0 QRC_CS_ARG);
                } else {
                    // Exactly once: the first CTA to set the mark owns the
                    // share.  Warp 0 waits for the claim; the other warps
                    // read the share into its own accumulator meanwhile, and
                    // it is dropped if the claim was lost.
                    __shared__ qrc_u32 s_lost;
                    if (threadIdx.x == 0) {
                        const qrc_u32 tag = __ldcg(&map[H_EPOCH]) + 1u;
                        s_lost = atomicExch(&map[O_CLAIMS + 128 * cm.side + own_k], tag) == tag;
                    }
#ifdef QRC_CHECKED
                    // coverage counts only the reads whose values are kept
                    CheckState cs_all = cs;
                    cs.bytes = 0; cs.xr = 0;
#endif
                    typename Op::Acc part = plain ? read_share<Op, 0>(Op::zero(), cm, sh, cm.side, own_k, pw0 QRC_CS_ARG)
                                                  : read_share<Op>(Op::zero(), cm, sh, cm.side, own_k, pw0 QRC_CS_ARG);
                    __syncthreads();                              // s_lost: another CTA of this launch had it
                    if (!s_lost) acc = Op::merge(acc, part);
#ifdef QRC_CHECKED
                    if (s_lost) { cs.bytes = cs_all.bytes; cs.xr = cs_all.xr; }
                    else { cs.bytes += cs_all.bytes; cs.xr ^= cs_all.xr; }
#endif
                }
            }
            if (tail) acc = read_tail<Op>(acc, cm, sh.R, map, cm.side, first QRC_CS_ARG);
        } else {
            SideWalk w;
            w.setup(a, end, map, mode);
#ifndef QRC_CHECKED
            if (S >= 2) {
                acc = bulk_walk<Op>(acc, w, S, map, lane, warp);
            } else
#endif
            {
                const int n512 = (int)(w.C >> 9);
                w.begin(lane);
#if QRC_ACROSS
                for (;;) {
                    qrc_u64 ch[8];
                    int m = 0;
                    #pragma unroll
                    for (int u = 0; u < 8; u++) {
                        ch[u] = (m == u) ? w.next(lane) : 0ull;
                        if (ch[u]) m++;
                    }
                    if (m == 0) break;
                    acc = chunks_across<Op>(acc, ch, m, n512, lane QRC_CS_ARG);
                    if (m < 8) break;
                }
#else
                for (qrc_u64 chunk = w.next(lane); chunk; chunk = w.next(lane))
                    acc = chunk_warp<Op>(acc, chunk, n512, lane QRC_CS_ARG);
#endif
            }
#if QRC_TIMELINE
            stolen = w.stolen;
#endif
        }
        griddep_launch_dependents();
#if QRC_TIMELINE
        {
            __shared__ qrc_u32 s_stolen;
            if (threadIdx.x == 0) s_stolen = 0;
            __syncthreads();
            if (lane == 0 && stolen) atomicAdd(&s_stolen, stolen);
            __syncthreads();
            qrc_u64 t_end;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_end));
            if (threadIdx.x == 0 && blockIdx.x < 256) {
                qrc_u32* tl = map + O_TIMELINE + 4 * blockIdx.x;
                tl[0] = (qrc_u32)t_start; tl[1] = (qrc_u32)t_end;
                tl[2] = (qrc_u32)cm.side | (s_stolen << 1); tl[3] = smid();
            }
        }
#endif
    }
    // Edges shorter than the body granule: head by CTA 0 warp 0, tail by the
    // last CTA's last warp.
    if (blockIdx.x == 0 && warp == 0) acc = edge_warp<Op>(acc, a, lo, lane QRC_CS_ARG);
    if (blockIdx.x == gridDim.x - 1 && warp == W - 1) acc = edge_warp<Op>(acc, hi, end, lane QRC_CS_ARG);
#ifdef QRC_CHECKED
    cov_flush(cs, lane, map);
#endif

    // ---- finish: block value, one global reduction, ticket ----------------
    const typename Fin::Red v = Fin::block(Op::to_red(acc));
    __shared__ int s_last;
    if (threadIdx.x == 0) {
        qrc_u32 t;
        if (Op::kIdempotent && sh.on && s_mark) map[s_mark] = s_tag;   // ordered before the ticket
#if QRC_FINISH == 1
        // The block's value goes out as a fire-and-forget reduction; the
        // ticket increment has release semantics (ordered after it) and
        // acquire semantics (the last CTA then sees every other CTA's
        // reduction and share mark).
        Fin::red(map, v);
        asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;"
                     : "=r"(t) : "l"(&map[H_RUN_TICKET]), "r"(gridDim.x - 1) : "memory");
#else
        Fin::red(map, v);
        __threadfence();
        t = atomicInc(&map[H_RUN_TICKET], gridDim.x - 1);
        __threadfence();
#endif
        s_last = (t == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;

    // ---- last CTA: unmarked shares, then publish ---------------------------
    // Warp 1 takes the accumulator while warp 0 loads the share marks: one
    // round trip for both (the same warp would stall on the exchange's reply
    // before issuing the mark loads).  Only a missing share costs more.
    __shared__ typename Fin::Red s_acc;
    __shared__ qrc_u32 s_wait_err;
    __shared__ int s_share;
    if (threadIdx.x == (blockDim.x > 32 ? 32u : 0u)) {
        s_acc = Fin::take(map);
        s_wait_err = __ldcg(&map[H_WAIT_ERR]);
    }
    typename Op::Acc acc2 = Op::zero();
    bool extra = false;
    if (sh.on) {
        for (;;) {
            if (warp == 0) {
                qrc_u32 mark[8];                  // all 256 marks in one round trip
                #pragma unroll
                for (int t = 0; t < 8; t++) mark[t] = __ldcg(&map[O_CLAIMS + 32 * t + lane]);
                int found = -1;
                #pragma unroll
                for (int t = 7; t >= 0; t--) {
                    const int k = (32 * t + lane) & 127;
                    const unsigned m = __ballot_sync(0xFFFFFFFFu, (qrc_u32)k < sh.sms(t >> 2) && mark[t] != s_tag);
                    if (m) found = 32 * t + __ffs(m) - 1;
                }
                if (lane == 0) {
                    s_share = found;
                    if (found >= 0) map[O_CLAIMS + found] = s_tag;
                }
            }
            __syncthreads();
            const int pick = s_share;
            __syncthreads();
            if (pick < 0) break;
            extra = true;
            ChunkMap cm;                      // only when a share was missed
            cm.setup(a, end, map, mode);
            acc2 = read_share<Op>(acc2, cm, sh, pick >> 7, pick & 127,
                                  share_first_page_word(cm, sh, pick >> 7, pick & 127, cm.page_bits[0]) QRC_CS_ARG);
        }
        if (threadIdx.x == 0) map[H_EPOCH] = s_tag;      // the next launch marks with s_tag + 1
#ifdef QRC_CHECKED
        cov_flush(cs, lane, map);
#endif
    } else {
        __syncthreads();
    }
    const typename Fin::Red v2 = extra ? Fin::block(Op::to_red(acc2)) : Fin::neutral();
    if (warp == 0) {                                  // the whole warp: the cross-GPU exchange uses every lane
        typename Fin::Red r = Fin::combine(s_acc, v2);
        const bool xchg_ok = xa.world > 1 ? Fin::exchange(xa, r, lane) : true;
        if (lane == 0) {
            map[H_QUEUE0] = 0u;
            map[H_QUEUE1] = 0u;
            bool err = s_wait_err != 0u;
            if (!xchg_ok) {
                err = true;
                map[H_XCHG_ERR] = 1u;
            }
            // a bounded wait that gave up leaves no valid result: NaN
            Op::publish(out, scale_out, r, err);
#if QRC_TIMELINE
            qrc_u64 t_fin;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_fin));
            map[O_TIMELINE + 1023] = (qrc_u32)t_fin;  // end of the launch's last CTA
#endif
        }
    }
}

}  // namespace qrc

#ifndef QRC_NO_PLUGIN_ABI
// ---------------------------------------------------------------------------
// QuickRunCUDA plugin ABI (QuickRunCUDA.cpp:408-411, :466-474)
// ---------------------------------------------------------------------------
extern "C" __global__ void __launch_bounds__(1024, 1)
init(float* A, unsigned int* side_map, float* C, int num_dwords, int arg1, int arg2) {
    (void)C; (void)arg1; (void)arg2;
    qrc::discover(A, num_dwords > 0 ? (qrc_u64)num_dwords * 4ull : 0ull, side_map);
}

// The operator is chosen when the file is compiled, as in the reference,
// whose reduction_op is edited in place (side_aware.cu:215-219):
// -H '#define QRC_PLUGIN_OP n' with n = 0 absmax (default), 1 max, 2 min,
// 3 sum, 4 sum of squares.  C[0] receives the result as a float (sums are
// accumulated in double and rounded once at the end).
#ifndef QRC_PLUGIN_OP
#define QRC_PLUGIN_OP 0
#endif
namespace qrc {
template <class Op>
struct FloatOut : Op {                 // a double result rounded to one float in C[0]
    QRC_DEV void publish(void* out, float* s, double r, bool err) {
        double d;
        Op::publish(&d, s, r, err);
        *(float*)out = (float)d;
    }
};
template <int K> struct PluginOp { typedef OpAbsF32 T; };
template <> struct PluginOp<1> { typedef OpMaxF32 T; };
template <> struct PluginOp<2> { typedef OpMinF32 T; };
template <> struct PluginOp<3> { typedef FloatOut<OpSumF32> T; };
template <> struct PluginOp<4> { typedef FloatOut<OpSumSqF32> T; };
}  // namespace qrc

extern "C" __global__ void __launch_bounds__(1024, 1)
kernel(float* A, unsigned int* side_map, float* C, int num_dwords, int mode, int arg2) {
    (void)arg2;
#if defined(FORCE_WRONG_SIDE)
    mode = (mode & qrc::SCHED_MASK) | qrc::MODE_WRONG_SIDE;
#elif defined(FORCE_RANDOM_SIDE)
    mode = (mode & qrc::SCHED_MASK) | qrc::MODE_IGNORE_PAGE_BITS;
#endif
    qrc::reduce_run<qrc::PluginOp<QRC_PLUGIN_OP>::T>(A, num_dwords > 0 ? (qrc_u64)num_dwords : 0ull, side_map, C,
                                                     nullptr, (qrc_u32)mode);
}
#endif  // QRC_NO_PLUGIN_ABI

#endif  // QRC_SIDE_AWARE_B200_CU
