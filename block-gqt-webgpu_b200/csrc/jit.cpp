// Layout-specialised decode attention: the kernel of attention_impl.cuh compiled at run time
// for the group structures of a launch's packed key heads (nibble dims, group offsets).  With
// the layout as compile-time constants every group and run loop of the dequant + QK phase
// unrolls, which removes the loop and per-group bookkeeping of the generic kernel; the
// arithmetic and its order are the same, so outputs are identical.  Heads with different
// structures get one inlined body each, chosen per CTA by its head index; their grid is
// (splits, sequences, heads), so the CTAs resident on an SM at one time mostly run one body
// (the usual (splits, heads, sequences) order ran every body on every SM at once and
// thrashed the instruction cache: twice the time).
//
// The toolkit's nvcc (run as a child process, device code only, the build's flags) compiles
// the package's own kernel source (csrc/, found next to this library) to an sm_100a cubin,
// loaded with cudaLibraryLoadData; about two seconds per distinct structure.  Without nvcc,
// NVRTC (loaded with dlopen) is the fallback: its kernels are correct but its headers declare
// some intrinsics differently, so they are a few percent slower than nvcc's.
// One kernel per key (dims, query rows, value type, the heads' structures), kept for the life
// of the process (at most kMaxEntries).  A key whose heads share one structure compiles on the
// launch that first needs it; a key with several is queued for background worker threads
// (host work only, no CUDA calls; at most kWorkers compiles at a time) while the generic
// kernel serves the launches.  The cubin is loaded by the first launch after that whose stream is not capturing
// a graph, or by bgtq_layout_jit_wait.  Anything that fails
// (no compiler, no sources, a compile or load error) leaves the generic kernel in use.
// BGTQ_LAYOUT_JIT=0 in the environment or bgtq_set_layout_jit(0) turns it off.
//
// Prebuilt kernels: bgtq_layout_jit_prebuild compiles a key's kernel ahead of time (the build
// does this for the structures of the benchmarked tables) into bgtq/aot/ next to the library,
// under a name made from the key and the kernel sources' contents.  A launch whose key has a
// prebuilt cubin there loads it at once instead of compiling, so a host without the toolkit
// still runs the specialised kernel; a cubin of other sources never matches a name.
#include <dlfcn.h>
#include <spawn.h>
#include <sys/wait.h>
#include <unistd.h>
#include <fcntl.h>
#include <cerrno>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <deque>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <sstream>
#include <map>
#include <mutex>
#include <string>
#include <sys/stat.h>
#include <thread>
#include <vector>

#include "bgtq_internal.h"

extern char **environ;

namespace bgtq {
namespace {

constexpr size_t kMaxEntries = 64;  // a cubin is a few hundred KB

typedef int (*nvrtcCreateProgram_t)(void **, const char *, const char *, int, const char *const *,
                                    const char *const *);
typedef int (*nvrtcCompileProgram_t)(void *, int, const char *const *);
typedef int (*nvrtcGetSize_t)(void *, size_t *);
typedef int (*nvrtcGetData_t)(void *, char *);
typedef int (*nvrtcDestroyProgram_t)(void **);

struct Nvrtc {
    bool ok = false;
    nvrtcCreateProgram_t create = nullptr;
    nvrtcCompileProgram_t compile = nullptr;
    nvrtcGetSize_t log_size = nullptr, cubin_size = nullptr;
    nvrtcGetData_t log = nullptr, cubin = nullptr;
    nvrtcDestroyProgram_t destroy = nullptr;
};

std::string cuda_home() {
    for (const char *v : {"CUDA_HOME", "CUDA_PATH"}) {
        const char *e = std::getenv(v);
        if (e && *e) return e;
    }
    return "/usr/local/cuda";
}

bool exists(const std::string &p) {
    struct stat st;
    return stat(p.c_str(), &st) == 0;
}

const Nvrtc &nvrtc() {
    static Nvrtc n;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = nullptr;
        for (const std::string &name : {std::string("libnvrtc.so.12"), std::string("libnvrtc.so"),
                                         cuda_home() + "/lib64/libnvrtc.so.12", cuda_home() + "/lib64/libnvrtc.so"}) {
            h = dlopen(name.c_str(), RTLD_NOW | RTLD_LOCAL);
            if (h) break;
        }
        if (!h) return;
        n.create = reinterpret_cast<nvrtcCreateProgram_t>(dlsym(h, "nvrtcCreateProgram"));
        n.compile = reinterpret_cast<nvrtcCompileProgram_t>(dlsym(h, "nvrtcCompileProgram"));
        n.log_size = reinterpret_cast<nvrtcGetSize_t>(dlsym(h, "nvrtcGetProgramLogSize"));
        n.log = reinterpret_cast<nvrtcGetData_t>(dlsym(h, "nvrtcGetProgramLog"));
        n.cubin_size = reinterpret_cast<nvrtcGetSize_t>(dlsym(h, "nvrtcGetCUBINSize"));
        n.cubin = reinterpret_cast<nvrtcGetData_t>(dlsym(h, "nvrtcGetCUBIN"));
        n.destroy = reinterpret_cast<nvrtcDestroyProgram_t>(dlsym(h, "nvrtcDestroyProgram"));
        n.ok = n.create && n.compile && n.log_size && n.log && n.cubin_size && n.cubin && n.destroy;
    });
    return n;
}

// csrc/ of this package: the library sits in bgtq/, the sources in ../csrc
std::string source_dir() {
    Dl_info info{};
    if (!dladdr(reinterpret_cast<void *>(&jit_set_enabled), &info) || !info.dli_fname) return "";
    std::string p(info.dli_fname);
    const size_t slash = p.find_last_of('/');
    p = slash == std::string::npos ? std::string(".") : p.substr(0, slash);
    for (const std::string dir : {p + "/../csrc", p + "/csrc"})
        if (exists(dir + "/attention_impl.cuh")) return dir;
    return "";
}

struct Entry {
    enum State { Compiling, Compiled, Ready, Failed } state = Compiling;
    std::vector<char> cubin;  // Compiled: waiting for a launch outside a capture to load it
    cudaLibrary_t lib = nullptr;
    cudaKernel_t kernel = nullptr;
};

// Never destroyed: a compile thread may still be running when the process exits.
std::mutex &g_mu = *new std::mutex;
std::map<std::string, Entry> &g_cache = *new std::map<std::string, Entry>;
std::atomic<int> g_enabled{-1};  // -1: not read from the environment yet
std::atomic<uint32_t> g_compiled{0}, g_built{0}, g_failed{0};  // cubins made, kernels loaded, failures

// Background compiles: a FIFO served by up to kWorkers threads (started as jobs arrive, never
// joined); g_cv signals both a queued job and a finished one.  Guarded by g_mu.
struct Job {
    JitKey key;
    std::string ks;
};
std::deque<Job> &g_queue = *new std::deque<Job>;
std::condition_variable &g_cv = *new std::condition_variable;
constexpr uint32_t kWorkers = 4;
uint32_t g_busy = 0;     // jobs queued or compiling
uint32_t g_workers = 0;  // worker threads started

bool same_layout(const JitLayout &x, const JitLayout &y) {
    if (x.ns != y.ns || x.ng != y.ng) return false;
    for (uint32_t g = 0; g <= x.ng; ++g)
        if (x.group_off[g] != y.group_off[g]) return false;
    return true;
}

// The distinct structures of the key's heads (in first-use order) and each head's index into them.
uint32_t layout_classes(const JitKey &k, uint32_t (&cls)[kMaxHeads], uint32_t (&first)[kMaxHeads]) {
    uint32_t n = 0;
    for (uint32_t h = 0; h < k.heads; ++h) {
        uint32_t c = 0;
        while (c < n && !same_layout(k.head[first[c]], k.head[h])) ++c;
        if (c == n) first[n++] = h;
        cls[h] = c;
    }
    return n;
}

// Heads with more than one structure: the kernel's grid is (splits, sequences, heads).
bool multi_layout(const JitKey &k) {
    uint32_t cls[kMaxHeads], first[kMaxHeads];
    return layout_classes(k, cls, first) > 1;
}

std::string key_string(const JitKey &k) {
    std::string s = std::to_string(k.D) + "/" + std::to_string(k.QM) + "/" + std::to_string(k.vf32) + "/" +
                    std::to_string(k.heads);
    for (uint32_t h = 0; h < k.heads; ++h) {
        const JitLayout &l = k.head[h];
        s += ";" + std::to_string(l.ns) + "/" + std::to_string(l.ng) + ":";
        for (uint32_t g = 0; g <= l.ng; ++g) s += std::to_string(l.group_off[g]) + ",";
    }
    return s;
}

// Changes whenever kernel_source below changes what it generates (it is part of the names of
// prebuilt cubins).
std::string kernel_source_marker() { return "bgtq_attn_jit/v1/"; }

std::string kernel_source(const JitKey &k) {
    uint32_t cls[kMaxHeads] = {}, first[kMaxHeads] = {};
    const uint32_t n = layout_classes(k, cls, first);
    const std::string D = std::to_string(k.D), QM = std::to_string(k.QM), VF = k.vf32 ? "true" : "false";
    std::string src = "#include \"attention_impl.cuh\"\n";
    for (uint32_t c = 0; c < n; ++c) {
        const JitLayout &l = k.head[first[c]];
        // go(g) as nested conditionals over g = 0 .. ng
        std::string go = "0u";
        for (int g = (int)l.ng; g >= 0; --g)
            go = "g == " + std::to_string(g) + "u ? " + std::to_string(l.group_off[g]) + "u : (" + go + ")";
        src += "struct JitGroups" + std::to_string(c) + " {\n"
               "    static constexpr bool kStatic = true;\n"
               "    static constexpr uint32_t kNG = " + std::to_string(l.ng) + "u, kNS = " + std::to_string(l.ns) + "u;\n"
               "    static __host__ __device__ constexpr uint32_t go(uint32_t g) { return " + go + "; }\n"
               "};\n";
    }
    src += "extern \"C\" __global__ void __launch_bounds__(bgtq::attn::kThreads, bgtq::attn::MinBlocks<" + D + ", " +
           QM + ", bgtq::KKind::Packed>::value)\n"
           "bgtq_attn_jit(const __grid_constant__ bgtq::AttnArgs a, const bgtq::attn::Plan pl, uint32_t d) {\n";
    // several structures: the grid is (splits, sequences, heads), so that the CTAs resident
    // on an SM at one time mostly run one head's body (instruction cache)
    if (n > 1) src += "    const uint32_t hd = blockIdx.z;\n";
    const std::string blk = n > 1 ? "blockIdx.x, hd, blockIdx.y" : "blockIdx.x, blockIdx.y, blockIdx.z";
    for (uint32_t c = 0; c < n; ++c) {
        std::string cond;
        for (uint32_t h = 0; h < k.heads; ++h)
            if (cls[h] == c) cond += std::string(cond.empty() ? "" : " || ") + "hd == " + std::to_string(h) + "u";
        const std::string body = "bgtq::attn::attn_body<" + D + ", " + QM + ", bgtq::KKind::Packed, " + VF +
                                 ", JitGroups" + std::to_string(c) + ">(a, pl, d, " + blk + ");\n";
        if (n == 1) src += "    " + body;
        else if (c + 1 < n) src += std::string(c ? "    else if (" : "    if (") + cond + ") " + body;
        else src += "    else " + body;
    }
    return src + "}\n";
}

// nvcc -cubin of `src` in a private temporary directory; false if nvcc is absent or fails.
bool nvcc_cubin(const std::string &src, const std::string &src_dir, std::vector<char> &cubin) {
    const std::string nvcc = cuda_home() + "/bin/nvcc";
    if (!exists(nvcc)) return false;
    const char *tmp = std::getenv("TMPDIR");
    std::string tmpl = std::string(tmp && *tmp ? tmp : "/tmp") + "/bgtq_jit_XXXXXX";
    std::vector<char> tbuf(tmpl.begin(), tmpl.end());
    tbuf.push_back('\0');
    if (!mkdtemp(tbuf.data())) return false;
    const std::string dir(tbuf.data()), cu = dir + "/k.cu", out = dir + "/k.cubin", log = dir + "/log.txt";
    bool ok = false;
    {
        std::ofstream f(cu);
        f << src;
    }
    std::vector<std::string> args = {nvcc, "-cubin", "-gencode", "arch=compute_100a,code=sm_100a", "-O3",
                                     "-std=c++17", "-I" + src_dir, "-o", out, cu};
    std::vector<char *> argv;
    for (auto &a : args) argv.push_back(&a[0]);
    argv.push_back(nullptr);
    posix_spawn_file_actions_t fa;
    posix_spawn_file_actions_init(&fa);
    posix_spawn_file_actions_addopen(&fa, 1, log.c_str(), O_WRONLY | O_CREAT | O_TRUNC, 0644);
    posix_spawn_file_actions_adddup2(&fa, 1, 2);
    pid_t pid = 0;
    if (posix_spawn(&pid, nvcc.c_str(), &fa, nullptr, argv.data(), environ) == 0) {
        int status = 0;
        while (waitpid(pid, &status, 0) < 0 && errno == EINTR) {
        }
        ok = WIFEXITED(status) && WEXITSTATUS(status) == 0;
    }
    posix_spawn_file_actions_destroy(&fa);
    if (ok) {
        std::ifstream f(out, std::ios::binary);
        std::stringstream ss;
        ss << f.rdbuf();
        const std::string b = ss.str();
        cubin.assign(b.begin(), b.end());
        ok = !cubin.empty();
    } else if (std::getenv("BGTQ_LAYOUT_JIT_LOG")) {
        std::ifstream f(log);
        std::stringstream ss;
        ss << f.rdbuf();
        std::fprintf(stderr, "bgtq layout JIT: nvcc failed:\n%s\n", ss.str().c_str());
    }
    for (const std::string &p : {cu, out, log}) unlink(p.c_str());
    rmdir(dir.c_str());
    return ok;
}

// ---- prebuilt (ahead-of-time) kernels ----
uint64_t fnv1a(const char *p, size_t n, uint64_t h = 1469598103934665603ull) {
    for (size_t i = 0; i < n; ++i) h = (h ^ (unsigned char)p[i]) * 1099511628211ull;
    return h;
}

bool read_file(const std::string &path, std::string &out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::stringstream ss;
    ss << f.rdbuf();
    out = ss.str();
    return true;
}

// The kernel sources every layout-specialised kernel is built from, hashed: prebuilt cubins
// are named with it, so only cubins of the current sources are found.  0 if unreadable.
uint64_t sources_digest() {
    static uint64_t digest = [] {
        const std::string dir = source_dir();
        if (dir.empty()) return (uint64_t)0;
        uint64_t h = 1469598103934665603ull;
        for (const char *f : {"attention_impl.cuh", "bgtq_internal.h"}) {
            std::string text;
            if (!read_file(dir + "/" + f, text)) return (uint64_t)0;
            h = fnv1a(text.data(), text.size(), h);
        }
        return h;
    }();
    return digest;
}

// bgtq/aot/ beside this library.
std::string aot_dir() {
    Dl_info info{};
    if (!dladdr(reinterpret_cast<void *>(&jit_set_enabled), &info) || !info.dli_fname) return "";
    std::string p(info.dli_fname);
    const size_t slash = p.find_last_of('/');
    return (slash == std::string::npos ? std::string(".") : p.substr(0, slash)) + "/aot";
}

// File name of a key's prebuilt cubin ("" when the sources cannot be read).
std::string aot_name(const std::string &ks) {
    const uint64_t d = sources_digest();
    if (!d) return "";
    const std::string src = kernel_source_marker() + ks;
    char buf[40];
    std::snprintf(buf, sizeof buf, "attn_%016llx.cubin", (unsigned long long)fnv1a(src.data(), src.size(), d));
    return buf;
}

std::atomic<uint32_t> g_prebuilt{0};  // keys served by a prebuilt cubin

bool load(Entry &e) {
    if (cudaLibraryLoadData(&e.lib, e.cubin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0) != cudaSuccess) {
        cudaGetLastError();
        e.lib = nullptr;
        return false;
    }
    if (cudaLibraryGetKernel(&e.kernel, e.lib, "bgtq_attn_jit") != cudaSuccess) {
        cudaGetLastError();
        cudaLibraryUnload(e.lib);
        e.lib = nullptr;
        return false;
    }
    return true;
}

// The key's kernel as an sm_100a cubin (host work only: nvcc, else NVRTC); empty on failure.
std::vector<char> compile(const JitKey &k) {
    std::vector<char> cubin;
    const std::string src_dir = source_dir(), inc = cuda_home() + "/include";
    if (src_dir.empty()) return cubin;
    const std::string src = kernel_source(k);
    if (nvcc_cubin(src, src_dir, cubin)) return cubin;
    cubin.clear();
    const Nvrtc &n = nvrtc();
    if (!n.ok || !exists(inc + "/cuda_fp16.h")) return cubin;
    void *prog = nullptr;
    if (n.create(&prog, src.c_str(), "bgtq_attn_jit.cu", 0, nullptr, nullptr) != 0) return cubin;
    const std::string i1 = "-I" + src_dir, i2 = "-I" + inc;
    const char *opts[] = {"--gpu-architecture=sm_100a", "-std=c++17", i1.c_str(), i2.c_str()};
    const int rc = n.compile(prog, 4, opts);
    if (rc == 0) {
        size_t sz = 0;
        if (n.cubin_size(prog, &sz) == 0 && sz) {
            cubin.resize(sz);
            if (n.cubin(prog, cubin.data()) != 0) cubin.clear();
        }
    } else if (std::getenv("BGTQ_LAYOUT_JIT_LOG")) {
        size_t sz = 0;
        n.log_size(prog, &sz);
        std::string log(sz, '\0');
        n.log(prog, &log[0]);
        std::fprintf(stderr, "bgtq layout JIT: compile failed:\n%s\n", log.c_str());
    }
    n.destroy(&prog);
    return cubin;
}

// A compiled entry's cubin moved into a library, or marked failed (caller holds g_mu).
void finish(Entry &e, std::vector<char> &&cubin) {
    e.cubin = std::move(cubin);
    e.state = e.cubin.empty() ? Entry::Failed : Entry::Compiled;
    (e.state == Entry::Failed ? g_failed : g_compiled).fetch_add(1);
}

void worker() {
    std::unique_lock<std::mutex> l(g_mu);
    for (;;) {
        g_cv.wait(l, [] { return !g_queue.empty(); });
        Job j = std::move(g_queue.front());
        g_queue.pop_front();
        l.unlock();
        std::vector<char> cubin = compile(j.key);
        l.lock();
        finish(g_cache[j.ks], std::move(cubin));
        --g_busy;
        g_cv.notify_all();
    }
}

// A compiled entry's library loaded (caller holds g_mu, outside any graph capture).
void load_compiled(Entry &e) {
    if (e.state != Entry::Compiled) return;
    if (load(e)) {
        e.state = Entry::Ready;
        g_built.fetch_add(1);
    } else {
        e.state = Entry::Failed;
        g_failed.fetch_add(1);
    }
    std::vector<char>().swap(e.cubin);
}

// 0 off, 1 every launch, 2 automatic (the default; BGTQ_LAYOUT_JIT=0 / 1 in the environment
// selects off / every launch)
int mode() {
    int v = g_enabled.load();
    if (v < 0) {
        const char *e = std::getenv("BGTQ_LAYOUT_JIT");
        v = e && e[0] == '0' ? 0 : e && e[0] == '1' ? 1 : 2;
        g_enabled.store(v);
    }
    return v;
}
bool enabled() { return mode() != 0; }

}  // namespace

void jit_set_enabled(int on) { g_enabled.store(on < 0 || on > 2 ? 2 : on); }
int jit_mode() { return mode(); }

namespace {
thread_local int t_suppressed = 0;
}
void jit_suppress_on_thread(int on) { t_suppressed = on; }

const void *jit_attention_kernel(const JitKey &key, cudaStream_t stream, bool *head_major) {
    *head_major = false;
    if (t_suppressed || !enabled() || key.heads < 1 || key.heads > (uint32_t)kMaxHeads) return nullptr;
    for (uint32_t h = 0; h < key.heads; ++h)
        if (key.head[h].ng < 1 || key.head[h].ng > (uint32_t)kMaxGroups) return nullptr;
    const std::string ks = key_string(key);
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_cache.find(ks);
    if (it == g_cache.end()) {
        if (g_cache.size() >= kMaxEntries) return nullptr;
        it = g_cache.emplace(ks, Entry{}).first;
        std::string pre;
        const std::string name = aot_name(ks);
        if (!name.empty() && read_file(aot_dir() + "/" + name, pre) && !pre.empty()) {
            finish(it->second, std::vector<char>(pre.begin(), pre.end()));
            g_prebuilt.fetch_add(1);
        } else if (!multi_layout(key)) {
            finish(it->second, compile(key));
        } else {
            g_queue.push_back(Job{key, ks});
            ++g_busy;
            if (g_workers < kWorkers && g_workers < g_busy) {
                std::thread(worker).detach();
                ++g_workers;
            }
            g_cv.notify_all();
            return nullptr;
        }
    }
    Entry &e = it->second;
    if (e.state == Entry::Compiled) {
        // loading is not a stream operation: keep it out of graph captures
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        if (cs != cudaStreamCaptureStatusNone) return nullptr;
        load_compiled(e);
    }
    if (e.state != Entry::Ready) return nullptr;
    *head_major = multi_layout(key);
    return reinterpret_cast<const void *>(e.kernel);
}

}  // namespace bgtq

extern "C" {

bgtq_status bgtq_set_layout_jit(int on) {
    bgtq::jit_set_enabled(on);
    return BGTQ_OK;
}

bgtq_status bgtq_layout_jit_stats(uint32_t *built, uint32_t *failed) {
    if (built) *built = bgtq::g_built.load();
    if (failed) *failed = bgtq::g_failed.load();
    return BGTQ_OK;
}

bgtq_status bgtq_layout_jit_wait(uint32_t timeout_ms) {
    std::unique_lock<std::mutex> l(bgtq::g_mu);
    const bool idle = bgtq::g_cv.wait_for(l, std::chrono::milliseconds(timeout_ms), [] { return bgtq::g_busy == 0; });
    for (auto &kv : bgtq::g_cache) bgtq::load_compiled(kv.second);
    return idle ? BGTQ_OK : BGTQ_ETIMEOUT;
}

bgtq_status bgtq_layout_jit_prebuilt(uint32_t *n) {
    if (!n) return BGTQ_EINVAL;
    *n = bgtq::g_prebuilt.load();
    return BGTQ_OK;
}

bgtq_status bgtq_layout_jit_prebuild(const char *dir, uint32_t heads, const uint32_t *const *configs,
                                     const size_t *n_configs, const float *const *tables, const size_t *n_tables,
                                     uint32_t rows, int v_f32, char *name_out, size_t name_capacity) {
    using namespace bgtq;
    if (!dir || !configs || !n_configs || !tables || !n_tables || heads < 1 || heads > (uint32_t)kMaxHeads ||
        rows < 1 || rows > (uint32_t)kMaxRows) {
        set_last_error("Invalid prebuild request");
        return BGTQ_EINVAL;
    }
    JitKey key{};
    uint32_t dim = 0;
    for (uint32_t h = 0; h < heads; ++h) {
        Layout L;
        std::string err;
        const bgtq_status st = parse_layout(configs[h], n_configs[h], tables[h], n_tables[h], L, err);
        if (st != BGTQ_OK) {
            set_last_error(err);
            return st;
        }
        if (h && L.d != dim) {
            set_last_error("Invalid prebuild request: heads of different dims");
            return BGTQ_EINVAL;
        }
        dim = L.d;
        key.head[h].ns = L.ns;
        key.head[h].ng = L.ng;
        for (uint32_t g = 0; g <= L.ng && g <= (uint32_t)kMaxGroups; ++g) key.head[h].group_off[g] = L.group_off[g];
    }
    key.D = dim <= 16 ? 16u : dim <= 32 ? 32u : dim <= 64 ? 64u : 128u;
    key.QM = attention_qm(KKind::Packed, rows);
    key.vf32 = v_f32 ? 1u : 0u;
    key.heads = heads;
    const std::string name = aot_name(key_string(key));
    if (name.empty()) {
        set_last_error("kernel sources not found next to the library");
        return BGTQ_ELAYOUT;
    }
    if (name_out && name_capacity) std::snprintf(name_out, name_capacity, "%s", name.c_str());
    const std::string path = std::string(dir) + "/" + name, tmp = path + ".tmp";
    if (exists(path)) return BGTQ_OK;  // built by an earlier run from the same sources
    std::vector<char> cubin = compile(key);
    if (cubin.empty()) {
        set_last_error("layout-specialised kernel did not compile (is nvcc installed?)");
        return BGTQ_ECUDA;
    }
    mkdir(dir, 0755);
    {
        std::ofstream f(tmp, std::ios::binary);
        f.write(cubin.data(), (std::streamsize)cubin.size());
        if (!f) {
            set_last_error("cannot write " + tmp);
            return BGTQ_EINVAL;
        }
    }
    if (std::rename(tmp.c_str(), path.c_str()) != 0) {
        set_last_error("cannot write " + path);
        return BGTQ_EINVAL;
    }
    return BGTQ_OK;
}

bgtq_status bgtq_layout_jit_counts(uint32_t *compiled, uint32_t *loaded, uint32_t *failed) {
    if (compiled) *compiled = bgtq::g_compiled.load();
    if (loaded) *loaded = bgtq::g_built.load();
    if (failed) *failed = bgtq::g_failed.load();
    return BGTQ_OK;
}

}  // extern "C"
