// qrc_harness.cpp -- B200 host harness for QuickRunCUDA kernel files.
//
// Mirrors the reference harness' run path for the side-aware reduction
// (QuickRunCUDA.cpp:354-658): it allocates A/B/C, compiles a kernel file with
// NVRTC (utils/cuda_helper.h:188-291) or loads a cubin, fills the arrays, runs
// `init` once (-i) and `kernel` once untimed plus -T timed times, and prints the
// same report line ("%.5f ms ==> %.4f GB/s ==> %.3f%%", QuickRunCUDA.cpp:559-576).
// Flag names and meanings follow QuickRunCUDA.cpp:132-195 for the subset this
// path uses.  Differences, all deliberate:
//   * NVRTC targets sm_100a by default (--arch sm_100 gives the reference's
//     choice, utils/cuda_helper.h:245, which adds `a` only for CC 9.0);
//   * --reference-c mismatches exit with status 1 (the reference only prints);
//   * --fill-a uniform:SEED[:OUTLIER] | normal:SEED[:SIGMA] fills A with the
//     seeded synthetic streams (the reference offers zeros or masked random
//     bits only); -r reproduces the reference's mt19937_64 fill bit for bit;
//   * --cubin FILE loads a prebuilt cubin (like --reuse-cubin with a path);
//   * --power-seconds S adds a time-based run with NVML power sampling
//     (the reference's NVML sampler exists but is never enabled,
//     QuickRunCUDA.cpp:291, utils/nvmlClass.h:275-302);
//   * --json prints one JSON object with the measurements;
//   * --dump-b FILE writes buffer B raw after the runs (kernel-file state);
//   * --clock-speed is not provided: this harness changes no GPU setting;
//   * --server [--server-dir D] keeps one process (and its CUDA context)
//     alive and runs command lines written to the FIFO D/quickruncuda_cmd
//     (D = /tmp by default, the reference's path), answering with the
//     command's standard output on D/quickruncuda_resp
//     (QuickRunCUDA.cpp:298-343, utils/ipc_helper.h).  "exit" ends it.  A
//     failing command answers with its error instead of ending the server,
//     and every command frees what it allocated.
// Errors print a message and exit non-zero (the reference exits from
// checkCudaErrors, utils/cuda_helper.h:17-33).
#include <cuda.h>
#include <nvrtc.h>
#include <nvml.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <random>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include "../csrc/qrc_gen.cuh"

#include <dlfcn.h>

// The driver API and NVML are loaded at run time (dlopen), so the binary also
// starts on machines without a GPU driver, where only --compile-only works.
#define QRC_XSTR(x) QRC_STR(x)
#define QRC_STR(x) #x
#define QRC_CU_FUNCS(X)                                                                        \
    X(cuInit) X(cuDeviceGet) X(cuDeviceGetAttribute) X(cuDevicePrimaryCtxRetain)                \
    X(cuDevicePrimaryCtxRelease) X(cuCtxSetCurrent) X(cuCtxSynchronize) X(cuMemAlloc)            \
    X(cuMemFree) X(cuMemcpyHtoD) X(cuMemcpyDtoH) X(cuMemsetD8) X(cuModuleLoadData)              \
    X(cuModuleUnload) X(cuModuleGetFunction) X(cuFuncSetAttribute) X(cuLaunchKernel)            \
    X(cuEventCreate) X(cuEventRecord) X(cuEventSynchronize) X(cuEventElapsedTime)               \
    X(cuEventDestroy) X(cuGetErrorName)
#define QRC_NVML_FUNCS(X)                                                                      \
    X(nvmlInit) X(nvmlShutdown) X(nvmlDeviceGetHandleByIndex) X(nvmlDeviceGetFieldValues)       \
    X(nvmlDeviceGetPowerUsage) X(nvmlDeviceGetClockInfo)

namespace dyn {
#define QRC_DECL(f) static decltype(&::f) p_##f = nullptr;
QRC_CU_FUNCS(QRC_DECL)
QRC_NVML_FUNCS(QRC_DECL)
#undef QRC_DECL

bool load_driver() {
    void* h = dlopen("libcuda.so.1", RTLD_NOW | RTLD_LOCAL);
    if (!h) return false;
#define QRC_LOAD(f) p_##f = reinterpret_cast<decltype(p_##f)>(dlsym(h, QRC_XSTR(f))); if (!p_##f) return false;
    QRC_CU_FUNCS(QRC_LOAD)
    return true;
}
bool load_nvml() {
    void* h = dlopen("libnvidia-ml.so.1", RTLD_NOW | RTLD_LOCAL);
    if (!h) return false;
    QRC_NVML_FUNCS(QRC_LOAD)
#undef QRC_LOAD
    return true;
}
}  // namespace dyn

namespace {

// In server mode an error ends the command, not the process.
bool g_server = false;
struct CommandError { std::string msg; int code; };

[[noreturn]] void die(const std::string& msg, int code = 2) {
    if (g_server) throw CommandError{msg, code};
    fprintf(stderr, "error: %s\n", msg.c_str());
    exit(code);
}

void ck(CUresult r, const char* what) {
    if (r != CUDA_SUCCESS) {
        const char* name = nullptr;
        dyn::p_cuGetErrorName(r, &name);
        die(std::string(what) + " failed: " + (name ? name : "?"));
    }
}
void ckr(nvrtcResult r, const char* what) {
    if (r != NVRTC_SUCCESS) die(std::string(what) + " failed: " + nvrtcGetErrorString(r));
}

struct Args {
    size_t dwordsA = 64ull << 20, dwordsB = 64ull << 20, dwordsC = 64ull << 20;
    bool randomA = false, randomB = false;
    unsigned randomMask = 0xFFFFFFFFu, randomSeed = 1234;
    int intArgs[3] = {0, 0, 0};
    int threads = 32, blocks = 1;
    bool persistent = false;
    int smemBytes = 0, carveout = 0;
    bool runInit = false;
    int l2flush = 0;
    int timedRuns = 0;
    float perfMult = 0.f, perfMultPerThread = 0.f, speedOfLight = 0.f;
    std::string unit = "ops/s";
    std::string kernelFile = "";
    std::string header = "";
    std::string cubinFile = "";
    std::string arch = "sm_100a";
    bool reuseCubin = false, timesPerRun = false, compileOnly = false, json = false;
    std::string dumpC, dumpCFormat = "raw", loadC, referenceC, dumpB;
    float compareTolerance = 0.f;
    std::string fillA;
    double powerSeconds = 0.0;
    int device = 0;
    bool server = false;
    std::string serverDir = "/tmp";
};

void usage() {
    printf(
        "qrc_harness -- run a QuickRunCUDA kernel file on a B200\n"
        "usage: qrc_harness [options] kernel.cu\n"
        "  -t,--threadsPerBlock N   -b,--blocksPerGrid N   -p,--persistentBlocks\n"
        "  -s,--sharedMemoryBlockBytes N   -o,--sharedMemoryCarveoutBytes N\n"
        "  -i,--runInitKernel   --l2flush 0|1|2\n"
        "  -T,--timedRuns N   -P,--perfMultiplier X   -N,--perfMultiplierPerThread X\n"
        "  -U,--perfMultiplier-unit S   -L,--perfSpeedOfLight X   --timesPerRun\n"
        "  -A/-B/-C,--arrayDwords{A,B,C} N   -r,--randomA   --randomB\n"
        "  --randomMask M (0x.. / 0b.. ok)   --randomSeed S\n"
        "  -0/-1/-2,--kernel-int-arg{0,1,2} V\n"
        "  -f,--kernel-filename F   -H,--header S   --reuse-cubin   --cubin F\n"
        "  --arch sm_100a|sm_100   --compile-only\n"
        "  --dump-c F   --dump-c-format raw|int_csv|float_csv   --load-c F   --dump-b F\n"
        "  --reference-c F   --compare-tolerance X\n"
        "  --fill-a uniform:SEED[:OUTLIER] | normal:SEED[:SIGMA]\n"
        "  --power-seconds S   --json   --device N\n"
        "  --server [--server-dir D]   (commands on D/quickruncuda_cmd, output on D/quickruncuda_resp)\n");
}

unsigned long long parse_u64(const std::string& s) {
    if (s.rfind("0x", 0) == 0 || s.rfind("0X", 0) == 0) return std::stoull(s.substr(2), nullptr, 16);
    if (s.rfind("0b", 0) == 0 || s.rfind("0B", 0) == 0) return std::stoull(s.substr(2), nullptr, 2);
    // accept 1e9-style sizes
    if (s.find_first_of("eE.") != std::string::npos) return (unsigned long long)std::llround(std::stod(s));
    return std::stoull(s, nullptr, 10);
}

Args parse(int argc, char** argv) {
    Args a;
    std::vector<std::string> pos;
    auto need = [&](int& i) -> std::string {
        if (i + 1 >= argc) die(std::string("missing value for ") + argv[i]);
        return argv[++i];
    };
    for (int i = 1; i < argc; i++) {
        std::string f = argv[i];
        if (f == "-h" || f == "--help") { usage(); if (g_server) die("", 0); exit(0); }
        else if (f == "-t" || f == "--threadsPerBlock") a.threads = std::stoi(need(i));
        else if (f == "-b" || f == "--blocksPerGrid") a.blocks = std::stoi(need(i));
        else if (f == "-p" || f == "--persistentBlocks") a.persistent = true;
        else if (f == "-s" || f == "--sharedMemoryBlockBytes") a.smemBytes = std::stoi(need(i));
        else if (f == "-o" || f == "--sharedMemoryCarveoutBytes") a.carveout = std::stoi(need(i));
        else if (f == "-i" || f == "--runInitKernel") a.runInit = true;
        else if (f == "--l2flush") a.l2flush = std::stoi(need(i));
        else if (f == "-T" || f == "--timedRuns") a.timedRuns = std::stoi(need(i));
        else if (f == "-P" || f == "--perfMultiplier") a.perfMult = std::stof(need(i));
        else if (f == "-N" || f == "--perfMultiplierPerThread") a.perfMultPerThread = std::stof(need(i));
        else if (f == "-U" || f == "--perfMultiplier-unit") a.unit = need(i);
        else if (f == "-L" || f == "--perfSpeedOfLight") a.speedOfLight = std::stof(need(i));
        else if (f == "--timesPerRun") a.timesPerRun = true;
        else if (f == "-A" || f == "--arrayDwordsA") a.dwordsA = parse_u64(need(i));
        else if (f == "-B" || f == "--arrayDwordsB") a.dwordsB = parse_u64(need(i));
        else if (f == "-C" || f == "--arrayDwordsC") a.dwordsC = parse_u64(need(i));
        else if (f == "-r" || f == "--randomA") a.randomA = true;
        else if (f == "--randomB") a.randomB = true;
        else if (f == "--randomMask") a.randomMask = (unsigned)parse_u64(need(i));
        else if (f == "--randomSeed") a.randomSeed = (unsigned)parse_u64(need(i));
        else if (f == "-0" || f == "--kernel-int-arg0") a.intArgs[0] = (int)(long long)parse_u64(need(i));
        else if (f == "-1" || f == "--kernel-int-arg1") a.intArgs[1] = std::stoi(need(i));
        else if (f == "-2" || f == "--kernel-int-arg2") a.intArgs[2] = std::stoi(need(i));
        else if (f == "-f" || f == "--kernel-filename") a.kernelFile = need(i);
        else if (f == "-H" || f == "--header") a.header = need(i);
        else if (f == "--reuse-cubin") a.reuseCubin = true;
        else if (f == "--cubin") a.cubinFile = need(i);
        else if (f == "--arch") a.arch = need(i);
        else if (f == "--compile-only") a.compileOnly = true;
        else if (f == "--dump-c") a.dumpC = need(i);
        else if (f == "--dump-c-format") a.dumpCFormat = need(i);
        else if (f == "--dump-b") a.dumpB = need(i);
        else if (f == "--load-c") a.loadC = need(i);
        else if (f == "--reference-c") a.referenceC = need(i);
        else if (f == "--compare-tolerance") a.compareTolerance = std::stof(need(i));
        else if (f == "--fill-a") a.fillA = need(i);
        else if (f == "--power-seconds") a.powerSeconds = std::stod(need(i));
        else if (f == "--json") a.json = true;
        else if (f == "--device") a.device = std::stoi(need(i));
        else if (f == "--clock-speed")
            die(f + " is not supported: this harness changes no GPU setting");
        else if (f == "--server") a.server = true;
        else if (f == "--server-dir") a.serverDir = need(i);
        else if (!f.empty() && f[0] == '-' && f.size() > 1) die("unknown option " + f);
        else pos.push_back(f);
    }
    if (!pos.empty()) a.kernelFile = pos[0];
    if (a.arch != "sm_100a" && a.arch != "sm_100") die("--arch must be sm_100a or sm_100");
    if (a.dumpCFormat != "raw" && a.dumpCFormat != "int_csv" && a.dumpCFormat != "float_csv")
        die("--dump-c-format must be raw, int_csv or float_csv");
    return a;
}

std::string read_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) die("cannot open " + path);
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

// NVRTC compile with the reference's options (utils/cuda_helper.h:223-253):
// header prepended, line info, fast math, C++17, the CUDA include path.
std::vector<char> compile_cubin(const Args& a) {
    if (a.kernelFile.empty()) die("no kernel file given");
    std::string src = a.header + "\n" + read_file(a.kernelFile);
    nvrtcProgram prog;
    ckr(nvrtcCreateProgram(&prog, src.c_str(), a.kernelFile.c_str(), 0, nullptr, nullptr), "nvrtcCreateProgram");
    std::string archOpt = "--gpu-architecture=" + a.arch;
    const char* cudaInc = getenv("CUDA_HOME");
    std::string inc = std::string("-I") + (cudaInc ? cudaInc : "/usr/local/cuda") + "/include";
    const char* opts[] = {"--generate-line-info", "-use_fast_math", "--std=c++17", archOpt.c_str(), inc.c_str()};
    nvrtcResult res = nvrtcCompileProgram(prog, 5, opts);
    size_t logSize = 0;
    nvrtcGetProgramLogSize(prog, &logSize);
    if (logSize > 2) {
        std::string log(logSize, '\0');
        nvrtcGetProgramLog(prog, &log[0]);
        fprintf(stderr, "\n------- NVRTC LOG -------\n%s\n------- END LOG -------\n", log.c_str());
    }
    ckr(res, "nvrtcCompileProgram");
    size_t n = 0;
    ckr(nvrtcGetCUBINSize(prog, &n), "nvrtcGetCUBINSize");
    std::vector<char> cubin(n);
    ckr(nvrtcGetCUBIN(prog, cubin.data()), "nvrtcGetCUBIN");
    nvrtcDestroyProgram(&prog);
    return cubin;
}

// The reference's -r fill (QuickRunCUDA.cpp:432-457): chunk c of 1 Mi dwords
// draws from std::mt19937_64(seed + c) through uniform_int_distribution<uint>,
// A's dwords first, then B's, each masked.
void fill_random(std::vector<uint32_t>& hA, std::vector<uint32_t>& hB, const Args& a) {
    const size_t chunk = 1024 * 1024;
    const size_t na = a.randomA ? a.dwordsA : 0, nb = a.randomB ? a.dwordsB : 0;
    const size_t nchunks = (std::max(a.dwordsA, a.dwordsB) + chunk - 1) / chunk;
    #pragma omp parallel for schedule(static)
    for (size_t c = 0; c < nchunks; c++) {
        std::mt19937_64 rng(a.randomSeed + c);
        std::uniform_int_distribution<unsigned> dist;
        size_t end = std::min((c + 1) * chunk, na);
        for (size_t i = c * chunk; i < end; ++i) hA[i] = dist(rng) & a.randomMask;
        end = std::min((c + 1) * chunk, nb);
        for (size_t i = c * chunk; i < end; ++i) hB[i] = dist(rng) & a.randomMask;
    }
}

void fill_synthetic(std::vector<uint32_t>& hA, const std::string& spec) {
    // uniform:SEED[:OUTLIER] or normal:SEED[:SIGMA]
    std::vector<std::string> parts;
    std::stringstream ss(spec);
    std::string p;
    while (std::getline(ss, p, ':')) parts.push_back(p);
    if (parts.size() < 2) die("--fill-a needs dist:seed");
    const uint64_t seed = parse_u64(parts[1]);
    const uint64_t key = qrc_gen::key_of(seed);
    float* x = reinterpret_cast<float*>(hA.data());
    const size_t n = hA.size();
    if (parts[0] == "uniform") {
        #pragma omp parallel for schedule(static)
        for (size_t i = 0; i < n; i++) x[i] = qrc_gen::uniform_pm1(key, i);
        if (parts.size() > 2 && n) {
            const float mag = std::stof(parts[2]);
            x[qrc_gen::outlier_index(seed, n)] = (float)qrc_gen::outlier_sign(seed) * mag;
        }
    } else if (parts[0] == "normal") {
        const float sigma = parts.size() > 2 ? std::stof(parts[2]) : 1.0f;
        #pragma omp parallel for schedule(static)
        for (size_t i = 0; i < n; i++) x[i] = qrc_gen::normal01(key, i) * sigma;
    } else {
        die("--fill-a distribution must be uniform or normal");
    }
}

// NVML power sampler (read-only queries; changes nothing on the GPU).
struct PowerSampler {
    nvmlDevice_t dev{};
    bool ok = false;
    std::atomic<bool> run{false};
    std::thread th;
    std::vector<std::pair<double, unsigned>> samples;   // (seconds since start, mW)
    std::vector<unsigned> clocks;
    explicit PowerSampler(int index) {
        if (!dyn::load_nvml()) return;
        if (dyn::p_nvmlInit() != NVML_SUCCESS) return;
        ok = dyn::p_nvmlDeviceGetHandleByIndex((unsigned)index, &dev) == NVML_SUCCESS;
    }
    ~PowerSampler() { stop(); if (ok) dyn::p_nvmlShutdown(); }
    void start() {
        if (!ok) return;
        run = true;
        th = std::thread([this] {
            auto t0 = std::chrono::steady_clock::now();
            while (run) {
                nvmlFieldValue_t fv{};
                fv.fieldId = NVML_FI_DEV_POWER_INSTANT;
                unsigned mw = 0, clk = 0;
                if (dyn::p_nvmlDeviceGetFieldValues(dev, 1, &fv) == NVML_SUCCESS && fv.nvmlReturn == NVML_SUCCESS)
                    mw = fv.value.uiVal;
                else
                    dyn::p_nvmlDeviceGetPowerUsage(dev, &mw);
                dyn::p_nvmlDeviceGetClockInfo(dev, NVML_CLOCK_SM, &clk);
                const double t = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
                samples.emplace_back(t, mw);
                clocks.push_back(clk);
                std::this_thread::sleep_for(std::chrono::milliseconds(10));
            }
        });
    }
    void stop() {
        if (th.joinable()) { run = false; th.join(); }
    }
    // Mean power over samples after `skip` seconds.
    double mean_watts(double skip) const {
        double s = 0; size_t n = 0;
        for (auto& p : samples) if (p.first >= skip && p.second) { s += p.second; n++; }
        return n ? s / n / 1000.0 : 0.0;
    }
    double median_clock(double skip) const {
        std::vector<unsigned> v;
        for (size_t i = 0; i < samples.size(); i++) if (samples[i].first >= skip && clocks[i]) v.push_back(clocks[i]);
        if (v.empty()) return 0;
        std::sort(v.begin(), v.end());
        return v[v.size() / 2];
    }
};


// Releases what one run allocated, also when an error ends it early.
struct RunResources {
    CUdeviceptr dA = 0, dB = 0, dC = 0, dFlush = 0;
    CUmodule mod = nullptr;
    CUdevice dev = 0;
    bool ctx = false;
    ~RunResources() {
        if (!ctx) return;
        dyn::p_cuCtxSynchronize();
        if (dA) dyn::p_cuMemFree(dA);
        if (dB) dyn::p_cuMemFree(dB);
        if (dC) dyn::p_cuMemFree(dC);
        if (dFlush) dyn::p_cuMemFree(dFlush);
        if (mod) dyn::p_cuModuleUnload(mod);
        dyn::p_cuDevicePrimaryCtxRelease(dev);
    }
};

int run_once(Args a) {
    if (a.compileOnly) {
        std::vector<char> cubin = compile_cubin(a);
        printf("compiled %s for %s: %zu bytes\n", a.kernelFile.c_str(), a.arch.c_str(), cubin.size());
        return 0;
    }

    if (!dyn::load_driver()) die("cannot load libcuda.so.1 (no GPU driver on this machine)");
    ck(dyn::p_cuInit(0), "cuInit");
    RunResources res;
    CUdevice& dev = res.dev;
    ck(dyn::p_cuDeviceGet(&dev, a.device), "cuDeviceGet");
    CUcontext ctx;
    ck(dyn::p_cuDevicePrimaryCtxRetain(&ctx, dev), "cuDevicePrimaryCtxRetain");
    res.ctx = true;
    ck(dyn::p_cuCtxSetCurrent(ctx), "cuCtxSetCurrent");

    const size_t sizeA = a.dwordsA * 4, sizeB = a.dwordsB * 4, sizeC = a.dwordsC * 4;
    CUdeviceptr& dA = res.dA;
    CUdeviceptr& dB = res.dB;
    CUdeviceptr& dC = res.dC;
    CUdeviceptr& dFlush = res.dFlush;
    ck(dyn::p_cuMemAlloc(&dA, std::max<size_t>(sizeA, 4)), "cuMemAlloc A");
    ck(dyn::p_cuMemAlloc(&dB, std::max<size_t>(sizeB, 4)), "cuMemAlloc B");
    ck(dyn::p_cuMemAlloc(&dC, std::max<size_t>(sizeC, 4)), "cuMemAlloc C");
    std::vector<uint32_t> hC(a.dwordsC);

    if (a.persistent) {
        ck(dyn::p_cuDeviceGetAttribute(&a.blocks, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, dev), "attribute");
        if (!a.json) printf("Using persistent blocks (%d = 1 per SM)\n", a.blocks);
    }

    std::vector<char> cubin;
    if (!a.cubinFile.empty() || a.reuseCubin) {
        std::string path = a.cubinFile.empty() ? "output.cubin" : a.cubinFile;
        std::string s = read_file(path);
        cubin.assign(s.begin(), s.end());
    } else {
        cubin = compile_cubin(a);
        std::ofstream o("output.cubin", std::ios::binary);
        if (o) o.write(cubin.data(), (std::streamsize)cubin.size());
    }
    CUmodule& mod = res.mod;
    ck(dyn::p_cuModuleLoadData(&mod, cubin.data()), "cuModuleLoadData");
    CUfunction kfn, ifn = nullptr;
    ck(dyn::p_cuModuleGetFunction(&kfn, mod, "kernel"), "dyn::p_cuModuleGetFunction(kernel)");
    if (a.runInit) ck(dyn::p_cuModuleGetFunction(&ifn, mod, "init"), "dyn::p_cuModuleGetFunction(init)");

    // C: load or zero (QuickRunCUDA.cpp:413-429).
    if (!a.loadC.empty()) {
        std::string s = read_file(a.loadC);
        if (s.size() != sizeC) die("--load-c file size does not match -C");
        ck(dyn::p_cuMemcpyHtoD(dC, s.data(), sizeC), "cuMemcpyHtoD C");
    } else {
        ck(dyn::p_cuMemsetD8(dC, 0, std::max<size_t>(sizeC, 4)), "cuMemsetD8 C");
    }
    // A / B (QuickRunCUDA.cpp:431-463).
    const bool hostA = a.randomA || !a.fillA.empty();
    if (hostA || a.randomB) {
        std::vector<uint32_t> hA(hostA ? a.dwordsA : 0), hB(a.randomB ? a.dwordsB : 0);
        if (a.randomA || a.randomB) fill_random(hA, hB, a);
        if (!a.fillA.empty()) fill_synthetic(hA, a.fillA);
        if (!hA.empty()) ck(dyn::p_cuMemcpyHtoD(dA, hA.data(), sizeA), "cuMemcpyHtoD A");
        if (!hB.empty()) ck(dyn::p_cuMemcpyHtoD(dB, hB.data(), sizeB), "cuMemcpyHtoD B");
    }
    if (!hostA) ck(dyn::p_cuMemsetD8(dA, 0, std::max<size_t>(sizeA, 4)), "cuMemsetD8 A");
    if (!a.randomB) ck(dyn::p_cuMemsetD8(dB, 0, std::max<size_t>(sizeB, 4)), "cuMemsetD8 B");

    int iargs[3] = {a.intArgs[0], a.intArgs[1], a.intArgs[2]};
    void* kargs[] = {&dA, &dB, &dC, &iargs[0], &iargs[1], &iargs[2]};
    auto flush = [&] {
        const size_t fl = 256ull << 20;
        if (!dFlush) ck(dyn::p_cuMemAlloc(&dFlush, fl), "cuMemAlloc flush");
        ck(dyn::p_cuMemsetD8(dFlush, 0, fl), "flush");
    };
    auto launch = [&](CUfunction f) {
        ck(dyn::p_cuLaunchKernel(f, a.blocks, 1, 1, a.threads, 1, 1, a.smemBytes, 0, kargs, nullptr), "cuLaunchKernel");
    };

    double initMs = 0.0;
    if (a.runInit) {
        ck(dyn::p_cuFuncSetAttribute(ifn, CU_FUNC_ATTRIBUTE_PREFERRED_SHARED_MEMORY_CARVEOUT, a.carveout), "carveout");
        ck(dyn::p_cuFuncSetAttribute(ifn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, a.smemBytes), "smem");
        CUevent e0, e1;
        ck(dyn::p_cuEventCreate(&e0, CU_EVENT_DEFAULT), "event");
        ck(dyn::p_cuEventCreate(&e1, CU_EVENT_DEFAULT), "event");
        ck(dyn::p_cuEventRecord(e0, nullptr), "record");
        launch(ifn);
        ck(dyn::p_cuEventRecord(e1, nullptr), "record");
        ck(dyn::p_cuEventSynchronize(e1), "init");
        float ms = 0;
        dyn::p_cuEventElapsedTime(&ms, e0, e1);
        initMs = ms;
        dyn::p_cuEventDestroy(e0); dyn::p_cuEventDestroy(e1);
    }
    if (a.l2flush >= 1) flush();
    ck(dyn::p_cuFuncSetAttribute(kfn, CU_FUNC_ATTRIBUTE_PREFERRED_SHARED_MEMORY_CARVEOUT, a.carveout), "carveout");
    ck(dyn::p_cuFuncSetAttribute(kfn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, a.smemBytes), "smem");
    launch(kfn);
    if (a.l2flush == 1) flush();
    ck(dyn::p_cuCtxSynchronize(), "warm-up kernel");

    float avgMs = 0.f, overallMs = 0.f;
    double perf = 0.0;
    std::vector<float> runTimes;
    if (a.timedRuns > 0) {
        const bool indiv = a.l2flush >= 2 || a.timesPerRun;
        CUevent os, oe;
        ck(dyn::p_cuEventCreate(&os, CU_EVENT_DEFAULT), "event");
        ck(dyn::p_cuEventCreate(&oe, CU_EVENT_DEFAULT), "event");
        std::vector<CUevent> st(indiv ? a.timedRuns : 0), en(indiv ? a.timedRuns : 0);
        for (int i = 0; i < (int)st.size(); i++) {
            ck(dyn::p_cuEventCreate(&st[i], CU_EVENT_DEFAULT), "event");
            ck(dyn::p_cuEventCreate(&en[i], CU_EVENT_DEFAULT), "event");
        }
        ck(dyn::p_cuEventRecord(os, nullptr), "record");
        for (int i = 0; i < a.timedRuns; i++) {
            if (a.l2flush == 2) flush();
            if (indiv) ck(dyn::p_cuEventRecord(st[i], nullptr), "record");
            launch(kfn);
            if (indiv) ck(dyn::p_cuEventRecord(en[i], nullptr), "record");
        }
        ck(dyn::p_cuEventRecord(oe, nullptr), "record");
        ck(dyn::p_cuEventSynchronize(oe), "timed runs");
        float total = 0.f;
        for (int i = 0; i < (int)st.size(); i++) {
            float ms = 0.f;
            ck(dyn::p_cuEventElapsedTime(&ms, st[i], en[i]), "elapsed");
            runTimes.push_back(ms);
            total += ms;
        }
        ck(dyn::p_cuEventElapsedTime(&overallMs, os, oe), "elapsed");
        if (a.timesPerRun && !a.json) {
            printf("Individual runtimes: ");
            for (int i = 0; i < a.timedRuns; i++) printf("%.5f %s", runTimes[i], i < a.timedRuns - 1 ? " / " : "\n");
        }
        avgMs = (indiv ? total : overallMs) / a.timedRuns;
        float mult = a.perfMult;
        if (a.perfMultPerThread > 0.f) mult = a.perfMultPerThread * a.threads * a.blocks;
        if (mult > 0.f) perf = mult / (avgMs / 1000.0);
        if (!a.json) {
            printf("\n%.5f ms", avgMs);
            if (indiv) printf(" (%.5f ms including L2 flushes)", overallMs / a.timedRuns);
            if (mult > 0.f) {
                printf(" ==> %.4f %s", perf, a.unit.c_str());
                if (a.speedOfLight > 0.f) printf(" ==> %.3f%%", 100.0 * perf / a.speedOfLight);
            }
            printf("\n\n");
        }
        dyn::p_cuEventDestroy(os); dyn::p_cuEventDestroy(oe);
        for (size_t i = 0; i < st.size(); i++) { dyn::p_cuEventDestroy(st[i]); dyn::p_cuEventDestroy(en[i]); }
    }

    // Time-based run with NVML power sampling: launches back to back in
    // batches of 32 until `powerSeconds` have elapsed on the device clock.
    double powerW = 0.0, powerPerf = 0.0, powerMs = 0.0, powerClock = 0.0;
    size_t powerSamples = 0;
    if (a.powerSeconds > 0.0) {
        PowerSampler ps(a.device);
        CUevent e0, e1;
        ck(dyn::p_cuEventCreate(&e0, CU_EVENT_DEFAULT), "event");
        ck(dyn::p_cuEventCreate(&e1, CU_EVENT_DEFAULT), "event");
        ps.start();
        ck(dyn::p_cuEventRecord(e0, nullptr), "record");
        long launches = 0;
        auto t0 = std::chrono::steady_clock::now();
        while (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() < a.powerSeconds) {
            for (int k = 0; k < 32; k++) launch(kfn);
            launches += 32;
            ck(dyn::p_cuCtxSynchronize(), "power run");
        }
        ck(dyn::p_cuEventRecord(e1, nullptr), "record");
        ck(dyn::p_cuEventSynchronize(e1), "power run");
        ps.stop();
        float ms = 0.f;
        dyn::p_cuEventElapsedTime(&ms, e0, e1);
        powerMs = ms / launches;
        float mult = a.perfMult;
        if (a.perfMultPerThread > 0.f) mult = a.perfMultPerThread * a.threads * a.blocks;
        powerPerf = mult > 0.f ? mult / (powerMs / 1000.0) : 0.0;
        powerW = ps.mean_watts(0.5);
        powerClock = ps.median_clock(0.5);
        powerSamples = ps.samples.size();
        if (!a.json)
            printf("power run: %.2f s, %ld launches, %.5f ms ==> %.4f %s, mean power %.1f W, median SM clock %.0f MHz (%zu samples)\n",
                   ms / 1000.0, launches, powerMs, powerPerf, a.unit.c_str(), powerW, powerClock, powerSamples);
        dyn::p_cuEventDestroy(e0); dyn::p_cuEventDestroy(e1);
    }

    ck(dyn::p_cuCtxSynchronize(), "final sync");
    int status = 0;
    if (!a.dumpC.empty() || !a.referenceC.empty() || a.json) {
        ck(dyn::p_cuMemcpyDtoH(hC.data(), dC, sizeC), "cuMemcpyDtoH C");
    }
    if (!a.dumpC.empty()) {
        if (a.dumpCFormat == "raw") {
            std::ofstream o(a.dumpC, std::ios::binary);
            o.write(reinterpret_cast<const char*>(hC.data()), (std::streamsize)sizeC);
        } else {
            std::ofstream o(a.dumpC);
            for (size_t i = 0; i < a.dwordsC; i++) {
                if (hC[i] != 0) {
                    if (a.dumpCFormat == "int_csv") o << hC[i];
                    else { float f; memcpy(&f, &hC[i], 4); o << std::fixed << std::setprecision(2) << f; }
                }
                if (i + 1 < a.dwordsC) o << ",";
            }
        }
    }
    if (!a.dumpB.empty()) {
        // Raw dump of B after the last launch (for kernel files that keep
        // state there, e.g. the side map and its diagnostics).
        std::vector<uint32_t> hB(a.dwordsB);
        ck(dyn::p_cuMemcpyDtoH(hB.data(), dB, sizeB), "cuMemcpyDtoH B");
        std::ofstream o(a.dumpB, std::ios::binary);
        o.write(reinterpret_cast<const char*>(hB.data()), (std::streamsize)sizeB);
    }
    long firstDiff = -1;
    if (!a.referenceC.empty()) {
        std::string ref = read_file(a.referenceC);
        if (ref.size() != sizeC) die("reference file missing or wrong size");
        const uint32_t* r = reinterpret_cast<const uint32_t*>(ref.data());
        for (size_t i = 0; i < a.dwordsC; i++) {
            bool diff;
            float x, y;
            memcpy(&x, &hC[i], 4); memcpy(&y, &r[i], 4);
            if (a.compareTolerance > 0.f) diff = std::fabs(x - y) > a.compareTolerance;
            else diff = hC[i] != r[i];
            if (diff) {
                printf("First difference at index %zu: %u vs %u\nHex: %08x vs %08x\nFP32: %.4f vs %.4f\n",
                       i, hC[i], r[i], hC[i], r[i], x, y);
                firstDiff = (long)i;
                status = 1;
                break;
            }
        }
    }
    if (a.json) {
        uint32_t c0 = a.dwordsC ? hC[0] : 0;
        float c0f; memcpy(&c0f, &c0, 4);
        printf("{\"kernel\": \"%s\", \"blocks\": %d, \"threads\": %d, \"timed_runs\": %d, \"avg_ms\": %.6f, "
               "\"overall_ms\": %.6f, \"perf\": %.6f, \"unit\": \"%s\", \"init_ms\": %.4f, \"c0_bits\": %u, "
               "\"c0\": %.9g, \"first_diff\": %ld, \"power_w\": %.2f, \"power_perf\": %.4f, \"power_ms\": %.6f, "
               "\"power_clock_mhz\": %.0f, \"power_samples\": %zu}\n",
               a.cubinFile.empty() ? a.kernelFile.c_str() : a.cubinFile.c_str(), a.blocks, a.threads, a.timedRuns,
               avgMs, overallMs / std::max(1, a.timedRuns), perf, a.unit.c_str(), initMs, c0, c0f, firstDiff,
               powerW, powerPerf, powerMs, powerClock, powerSamples);
    }

    return status;                  // res frees the buffers and the module
}

// ---------------------------------------------------------------------------
// Server mode (QuickRunCUDA.cpp:298-343, utils/ipc_helper.h)
// ---------------------------------------------------------------------------

// A command line split on white space, with '...' grouping as in the
// reference's parseCommandString (QuickRunCUDA.cpp:198-240).
std::vector<std::string> split_command(const std::string& cmd) {
    std::vector<std::string> out{"qrc_harness"};
    std::string cur;
    bool quoted = false, have = false;
    for (char c : cmd) {
        if (c == '\'') {
            if (quoted) { out.push_back(cur); cur.clear(); have = false; }
            quoted = !quoted;
        } else if (quoted || !std::isspace((unsigned char)c)) {
            cur += c; have = true;
        } else if (have) {
            out.push_back(cur); cur.clear(); have = false;
        }
    }
    if (have) out.push_back(cur);
    return out;
}

std::string read_all(int fd) {
    std::string s;
    char buf[65536];
    ssize_t n;
    while ((n = read(fd, buf, sizeof(buf))) > 0) s.append(buf, (size_t)n);
    return s;
}

// Runs one command with stdout going to a temporary file (no pipe, so large
// outputs cannot block), and returns that output.
std::string run_captured(const std::string& cmd) {
    fflush(stdout);
    FILE* tmp = tmpfile();
    if (!tmp) return "error: cannot create a capture file\n";
    const int saved = dup(STDOUT_FILENO);
    dup2(fileno(tmp), STDOUT_FILENO);
    std::string err;
    try {
        std::vector<std::string> words = split_command(cmd);
        std::vector<char*> argv;
        for (auto& w : words) argv.push_back(&w[0]);
        Args a = parse((int)argv.size(), argv.data());
        if (a.server) die("--server inside a server command");
        run_once(a);
    } catch (const CommandError& e) {
        if (!e.msg.empty()) err = "error: " + e.msg + "\n";
    } catch (const std::exception& e) {
        err = std::string("error: ") + e.what() + "\n";
    }
    fflush(stdout);
    dup2(saved, STDOUT_FILENO);
    close(saved);
    std::string out;
    rewind(tmp);
    out = read_all(fileno(tmp));
    fclose(tmp);
    return out + err;
}

int serve(const Args& a) {
    g_server = true;
    const std::string cmdPath = a.serverDir + "/quickruncuda_cmd", respPath = a.serverDir + "/quickruncuda_resp";
    for (const auto& p : {cmdPath, respPath})
        if (mkfifo(p.c_str(), 0666) != 0 && errno != EEXIST) {
            fprintf(stderr, "error: cannot create %s: %s\n", p.c_str(), strerror(errno));
            return 2;
        }
    // Keep the primary context alive between commands when a GPU is present.
    CUdevice dev = 0;
    CUcontext ctx = nullptr;
    const bool gpu = dyn::load_driver() && dyn::p_cuInit(0) == CUDA_SUCCESS &&
                     dyn::p_cuDeviceGet(&dev, a.device) == CUDA_SUCCESS &&
                     dyn::p_cuDevicePrimaryCtxRetain(&ctx, dev) == CUDA_SUCCESS;
    for (;;) {
        const int fd = open(cmdPath.c_str(), O_RDONLY);
        if (fd < 0) break;
        std::string cmd = read_all(fd);
        close(fd);
        while (!cmd.empty() && std::isspace((unsigned char)cmd.back())) cmd.pop_back();
        if (cmd == "exit") break;
        if (cmd.empty()) continue;
        const std::string out = run_captured(cmd);
        const int wfd = open(respPath.c_str(), O_WRONLY);
        if (wfd < 0) break;
        for (size_t off = 0; off < out.size();) {
            const ssize_t n = write(wfd, out.data() + off, out.size() - off);
            if (n <= 0) break;
            off += (size_t)n;
        }
        close(wfd);
    }
    unlink(cmdPath.c_str());
    unlink(respPath.c_str());
    if (gpu) dyn::p_cuDevicePrimaryCtxRelease(dev);
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    Args a = parse(argc, argv);
    if (a.server) return serve(a);
    return run_once(a);
}
