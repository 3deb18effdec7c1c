// Hot-tier fill through pinned staging: how a missed expert's bytes get from a
// host source into its device slot on the copy stream.
//
// The reference (sabah/runtime/cuda/sabah_rt.cu:1033-1514, fill :2051-2116)
// reads misses from disk with unbuffered I/O into a double-buffered pinned
// staging pool and issues the host-to-device copy from there, in waves of
// SABAH_LLAMA_IO_DEPTH reads spread over reader lanes. This is the Linux
// counterpart:
//
// * A source in pinned host memory (cudaHostAlloc / cudaHostRegister) is
//   copied directly: the DMA engine reads it, nothing is staged.
// * Any other source (pageable memory, an mmapped GGUF) is cut into chunks of
//   at most 4 MiB. Reader lanes (SABAH_LLAMA_IO_WORKERS threads, default the
//   depth) each take a chunk, claim a staging buffer of the ring
//   (SABAH_LLAMA_IO_DEPTH buffers, default 8), wait on the buffer's event for
//   its previous copy to have landed, fill it, queue cudaMemcpyAsync from it
//   on the copy stream and record the buffer's event. Filling the next chunk
//   overlaps the DMA of the previous ones, and the device copy is a true
//   asynchronous DMA from pinned memory.
// * Filling: when the source lies in a file mapping (/proc/self/maps) and
//   direct I/O is on (SABAH_LLAMA_DIRECT_IO, default on; "0" or "off" turns it
//   off), the lane reads the file with O_DIRECT at the 4096-aligned range that
//   covers the chunk. Otherwise, or when that read cannot be made (a file
//   system without O_DIRECT, a short read), it copies from the mapping.
//
// The caller (the residency code in sb_runtime.cu) holds the residency lock,
// records the copy stream's completion event after sb_stage_fill returns, and
// makes the compute stream wait on it, as for direct copies.
//
// Staging readahead (SABAH_LLAMA_PREFETCH=1, off by default as in the
// reference, sabah_rt.cu:1517-1860): a layer's gate, up and down calls read the
// same router ids, so when the first of them has its ids, the experts the other
// two will miss are known. The residency code offers those experts here; 8
// reader threads read each into a pinned readahead buffer of its own (O_DIRECT
// from the file where the source is file-mapped). The bytes stay there: nothing
// is reserved in the hot tier, so a wrong guess costs a read and no slot. When
// the follower call misses the expert, sb_pf_take queues the copy straight from
// that buffer (waiting up to 50 ms for a read still in flight rather than
// reading the same bytes twice), and the buffer is reused once that copy has
// landed. With every buffer busy, an offer replaces the oldest unclaimed
// readahead, or is dropped.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "sb_staging.h"

namespace {

constexpr size_t kChunk = (size_t)4 << 20;   // bytes per staged copy
constexpr size_t kAlign = 4096;              // O_DIRECT offset / length / buffer alignment
constexpr int kMaxDepth = 32;

int env_int(const char* name, int def, int lo, int hi) {
    const char* v = std::getenv(name);
    long n = v ? std::strtol(v, nullptr, 10) : def;
    if (!v || n == 0) n = def;
    return (int)std::max<long>(lo, std::min<long>(hi, n));
}
bool direct_io_on() {
    const char* v = std::getenv("SABAH_LLAMA_DIRECT_IO");
    return !(v && (std::strcmp(v, "0") == 0 || std::strcmp(v, "off") == 0));
}

// file mappings of this process, looked up by address
struct Mapping {
    uintptr_t lo, hi;
    uint64_t off;     // file offset of lo
    int fd;           // O_DIRECT descriptor, -1 if the file cannot be opened that way
};

struct Chunk {
    void* dst;
    const uint8_t* src;
    size_t bytes;
    bool direct;      // try O_DIRECT (the wave's SABAH_LLAMA_DIRECT_IO)
};

struct Buffer {
    std::mutex mu;               // held from claim to event record: the next user waits for it
    uint8_t* mem = nullptr;      // pinned, kAlign-aligned, kChunk + 2 * kAlign bytes
    uint8_t* raw = nullptr;
    cudaEvent_t ev = nullptr;    // recorded after the copy out of this buffer
};

struct Stager {
    std::mutex mu;               // guards the queue, the pool state and the mapping cache
    std::condition_variable cv_work, cv_done;
    std::deque<Chunk> queue;
    int pending = 0;             // chunks queued or in progress in the current wave
    bool failed = false;
    std::string error;
    bool stop = false;
    std::vector<std::thread> lanes;
    Buffer buf[kMaxDepth];
    int depth = 0;
    std::atomic<unsigned> next{0};
    cudaStream_t copy = nullptr;
    int device = 0;
    std::vector<Mapping> maps;
    bool maps_loaded = false;
    std::map<std::string, int> fds;
    std::atomic<unsigned long long> staged_bytes{0}, pinned_bytes{0}, dio_reads{0}, dio_bytes{0}, dio_fallbacks{0},
        waves{0};
    // a process that never called sabah_rt_shutdown still stops its lanes at exit
    ~Stager() {
        {
            std::lock_guard<std::mutex> l(mu);
            stop = true;
        }
        cv_work.notify_all();
        for (std::thread& t : lanes)
            if (t.joinable()) t.join();
    }
};
Stager g_st;

// all file mappings of the process (/proc/self/maps), each file opened once with O_DIRECT
void load_maps_locked() {
    g_st.maps.clear();
    FILE* f = std::fopen("/proc/self/maps", "r");
    if (!f) return;
    char line[4096];
    while (std::fgets(line, sizeof(line), f)) {
        unsigned long lo, hi, foff, inode;
        char perms[8], dev[16];
        int consumed = 0;
        if (std::sscanf(line, "%lx-%lx %7s %lx %15s %lu %n", &lo, &hi, perms, &foff, dev, &inode, &consumed) < 6) continue;
        if (inode == 0 || consumed <= 0 || line[consumed] != '/') continue;
        std::string path(line + consumed);
        while (!path.empty() && (path.back() == '\n' || path.back() == ' ')) path.pop_back();
        auto it = g_st.fds.find(path);
        int fd;
        if (it != g_st.fds.end()) {
            fd = it->second;
        } else {
            fd = ::open(path.c_str(), O_RDONLY | O_DIRECT);
            g_st.fds[path] = fd;
        }
        g_st.maps.push_back({(uintptr_t)lo, (uintptr_t)hi, (uint64_t)foff, fd});
    }
    std::fclose(f);
    g_st.maps_loaded = true;
}

// the file mapping that holds [p, p + n), looked up in the cache and, on a
// miss, in a fresh read of /proc/self/maps
bool mapping_of(const void* p, size_t n, Mapping& out) {
    std::lock_guard<std::mutex> l(g_st.mu);
    for (int pass = 0; pass < 2; ++pass) {
        if (!g_st.maps_loaded || pass == 1) load_maps_locked();
        for (const Mapping& m : g_st.maps)
            if ((uintptr_t)p >= m.lo && (uintptr_t)p + n <= m.hi) {
                out = m;
                return true;
            }
    }
    return false;
}

// one chunk: claim a buffer, fill it (O_DIRECT read or copy from the mapping),
// queue its DMA on the copy stream, record the buffer's event
bool run_chunk(const Chunk& c, std::string& why) {
    Buffer& b = g_st.buf[g_st.next.fetch_add(1) % (unsigned)g_st.depth];
    std::lock_guard<std::mutex> l(b.mu);
    if (cudaEventSynchronize(b.ev) != cudaSuccess) {   // its previous copy has landed
        why = "staging event wait failed";
        return false;
    }
    const uint8_t* from = nullptr;
    if (c.direct) {
        Mapping m;
        if (mapping_of(c.src, c.bytes, m) && m.fd >= 0) {
            const uint64_t off = m.off + ((uintptr_t)c.src - m.lo);
            const uint64_t base = off & ~(uint64_t)(kAlign - 1);
            const size_t delta = (size_t)(off - base);
            const size_t len = (delta + c.bytes + kAlign - 1) & ~(kAlign - 1);
            const ssize_t got = ::pread(m.fd, b.mem, len, (off_t)base);
            if (got >= (ssize_t)(delta + c.bytes)) {
                from = b.mem + delta;
                ++g_st.dio_reads;
                g_st.dio_bytes += c.bytes;
            } else {
                ++g_st.dio_fallbacks;
            }
        }
    }
    if (!from) {
        std::memcpy(b.mem, c.src, c.bytes);
        from = b.mem;
    }
    if (cudaMemcpyAsync(c.dst, from, c.bytes, cudaMemcpyHostToDevice, g_st.copy) != cudaSuccess ||
        cudaEventRecord(b.ev, g_st.copy) != cudaSuccess) {
        why = "staged copy failed";
        return false;
    }
    g_st.staged_bytes += c.bytes;
    return true;
}

void lane_main() {
    cudaSetDevice(g_st.device);
    for (;;) {
        Chunk c;
        {
            std::unique_lock<std::mutex> l(g_st.mu);
            g_st.cv_work.wait(l, [] { return g_st.stop || !g_st.queue.empty(); });
            if (g_st.stop) return;
            c = g_st.queue.front();
            g_st.queue.pop_front();
        }
        std::string why;
        const bool ok = run_chunk(c, why);
        std::lock_guard<std::mutex> l(g_st.mu);
        if (!ok && !g_st.failed) {
            g_st.failed = true;
            g_st.error = why;
        }
        if (--g_st.pending == 0) g_st.cv_done.notify_all();
    }
}

bool start_locked(cudaStream_t copy) {
    if (g_st.depth > 0) return true;
    cudaGetDevice(&g_st.device);
    const int depth = env_int("SABAH_LLAMA_IO_DEPTH", 8, 1, kMaxDepth);
    for (int i = 0; i < depth; ++i) {
        Buffer& b = g_st.buf[i];
        if (cudaHostAlloc((void**)&b.raw, kChunk + 2 * kAlign, cudaHostAllocDefault) != cudaSuccess ||
            cudaEventCreateWithFlags(&b.ev, cudaEventDisableTiming) != cudaSuccess) {
            sb_set_error("staging ring allocation failed");
            return false;
        }
        b.mem = (uint8_t*)(((uintptr_t)b.raw + kAlign - 1) & ~(uintptr_t)(kAlign - 1));
    }
    g_st.depth = depth;
    g_st.copy = copy;
    const int workers = env_int("SABAH_LLAMA_IO_WORKERS", depth, 1, 16);
    g_st.stop = false;
    for (int i = 0; i < workers; ++i) g_st.lanes.emplace_back(lane_main);
    return true;
}

bool is_pinned(const void* p) {
    cudaPointerAttributes at{};
    const bool ok = cudaPointerGetAttributes(&at, p) == cudaSuccess;
    cudaGetLastError();
    return ok && at.type == cudaMemoryTypeHost;
}

}  // namespace

bool sb_stage_fill(const sb_fill* f, int n, cudaStream_t copy) {
    std::vector<Chunk> chunks;
    const bool direct = direct_io_on();
    for (int i = 0; i < n; ++i) {
        if (is_pinned(f[i].src)) {
            if (!sb_cuda_ok(cudaMemcpyAsync(f[i].dst, f[i].src, f[i].bytes, cudaMemcpyHostToDevice, copy),
                            "expert H2D"))
                return false;
            g_st.pinned_bytes += f[i].bytes;
            continue;
        }
        for (size_t o = 0; o < f[i].bytes; o += kChunk)
            chunks.push_back({(uint8_t*)f[i].dst + o, (const uint8_t*)f[i].src + o, std::min(kChunk, f[i].bytes - o),
                              direct});
    }
    if (chunks.empty()) return true;
    std::unique_lock<std::mutex> l(g_st.mu);
    if (!start_locked(copy)) return false;
    if (g_st.copy != copy) {
        sb_set_error("staged fill: the copy stream changed");
        return false;
    }
    g_st.failed = false;
    g_st.maps_loaded = false;   // address ranges may have been unmapped and reused since the last wave
    g_st.pending += (int)chunks.size();
    for (const Chunk& c : chunks) g_st.queue.push_back(c);
    ++g_st.waves;
    g_st.cv_work.notify_all();
    g_st.cv_done.wait(l, [] { return g_st.pending == 0; });
    if (g_st.failed) {
        sb_set_error("%s", g_st.error.c_str());
        return false;
    }
    return true;
}

// ------------------------------------------------------------ staging readahead
namespace {

constexpr int kPfBuffers = 8;          // readahead buffers = reads in flight
constexpr size_t kPfMaxQueue = 64;
constexpr int kPfWaitMs = 50;

enum PfState { kPfFree, kPfFilling, kPfReady, kPfTaken, kPfFail };

struct PfBuffer {
    uint8_t* raw = nullptr;
    uint8_t* mem = nullptr;        // pinned, kAlign-aligned
    size_t cap = 0;                // usable bytes at mem
    size_t delta = 0;              // the expert's bytes start at mem + delta
    int state = kPfFree;
    const void* src = nullptr;     // identity: the expert's host bytes
    size_t bytes = 0;
    uint64_t seq = 0;
    cudaEvent_t free_ev = nullptr; // recorded after the copy out of this buffer
    bool free_pending = false;
};

struct PfJob {
    int buf;
    const uint8_t* src;
    size_t bytes;
};

struct Prefetcher {
    std::mutex mu;
    std::condition_variable cv_work, cv_done;
    std::deque<PfJob> queue;
    PfBuffer buf[kPfBuffers];
    std::vector<std::thread> readers;
    bool stop = false;
    int device = 0;
    uint64_t seq = 0;
    unsigned long long reads = 0, read_bytes = 0, used = 0, used_bytes = 0, dropped = 0, stale = 0, waits = 0,
                       wait_ns = 0, wait_timeouts = 0;
    ~Prefetcher() {
        {
            std::lock_guard<std::mutex> l(mu);
            stop = true;
        }
        cv_work.notify_all();
        for (std::thread& t : readers)
            if (t.joinable()) t.join();
    }
};
Prefetcher g_pf;

bool pf_env_on() {
    static int on = -1;
    if (on < 0) {
        const char* v = std::getenv("SABAH_LLAMA_PREFETCH");
        on = v && *v && std::strcmp(v, "0") != 0 && std::strcmp(v, "off") != 0;
    }
    return on != 0;
}

// Room for `need` bytes, and no copy still reading the buffer. Reader thread,
// while the buffer is kPfFilling (nobody else touches it then).
bool pf_prepare(PfBuffer& b, size_t need) {
    if (b.free_pending) {
        if (cudaEventSynchronize(b.free_ev) != cudaSuccess) return false;
        b.free_pending = false;
    }
    if (b.cap < need) {
        if (b.raw) cudaFreeHost(b.raw);
        b.raw = b.mem = nullptr;
        b.cap = 0;
        if (cudaHostAlloc((void**)&b.raw, need + kAlign, cudaHostAllocDefault) != cudaSuccess) return false;
        b.mem = (uint8_t*)(((uintptr_t)b.raw + kAlign - 1) & ~(uintptr_t)(kAlign - 1));
        b.cap = need;
    }
    return true;
}

// One expert into its buffer: an O_DIRECT read of the covering aligned range
// when the bytes lie in a file mapping and direct I/O is on, else a copy from
// the source.
bool pf_read(PfBuffer& b, const uint8_t* src, size_t bytes) {
    if (direct_io_on()) {
        Mapping m;
        if (mapping_of(src, bytes, m) && m.fd >= 0) {
            const uint64_t off = m.off + ((uintptr_t)src - m.lo);
            const uint64_t base = off & ~(uint64_t)(kAlign - 1);
            const size_t delta = (size_t)(off - base);
            const size_t len = (delta + bytes + kAlign - 1) & ~(kAlign - 1);
            if (!pf_prepare(b, len)) return false;
            const ssize_t got = ::pread(m.fd, b.mem, len, (off_t)base);
            if (got >= (ssize_t)(delta + bytes)) {
                b.delta = delta;
                ++g_st.dio_reads;
                g_st.dio_bytes += bytes;
                return true;
            }
            ++g_st.dio_fallbacks;
        }
    }
    if (!pf_prepare(b, bytes)) return false;
    std::memcpy(b.mem, src, bytes);
    b.delta = 0;
    return true;
}

void pf_reader() {
    cudaSetDevice(g_pf.device);
    for (;;) {
        PfJob j;
        {
            std::unique_lock<std::mutex> l(g_pf.mu);
            g_pf.cv_work.wait(l, [] { return g_pf.stop || !g_pf.queue.empty(); });
            if (g_pf.stop) return;
            j = g_pf.queue.front();
            g_pf.queue.pop_front();
        }
        PfBuffer& b = g_pf.buf[j.buf];
        const bool ok = pf_read(b, j.src, j.bytes);
        {
            std::lock_guard<std::mutex> l(g_pf.mu);
            b.state = ok ? kPfReady : kPfFail;
            if (ok) {
                ++g_pf.reads;
                g_pf.read_bytes += j.bytes;
            }
        }
        g_pf.cv_done.notify_all();   // a miss may be waiting for this buffer
    }
}

void pf_start_locked() {
    if (!g_pf.readers.empty()) return;
    cudaGetDevice(&g_pf.device);
    g_pf.stop = false;
    for (int i = 0; i < kPfBuffers; ++i) g_pf.readers.emplace_back(pf_reader);
}

}  // namespace

bool sb_pf_enabled() { return pf_env_on(); }

void sb_pf_offer(const void* src, size_t bytes) {
    if (!pf_env_on() || !src || bytes == 0 || is_pinned(src)) return;
    std::lock_guard<std::mutex> l(g_pf.mu);
    pf_start_locked();
    if (g_pf.queue.size() >= kPfMaxQueue) return;
    int pick = -1;
    for (int i = 0; i < kPfBuffers; ++i) {
        const PfBuffer& b = g_pf.buf[i];
        if ((b.state == kPfReady || b.state == kPfFilling) && b.src == src && b.bytes == bytes) return;
        if (pick < 0 && (b.state == kPfFree || b.state == kPfFail)) pick = i;
    }
    if (pick < 0) {   // every buffer busy: the oldest readahead nobody has claimed
        uint64_t oldest = ~0ull;
        for (int i = 0; i < kPfBuffers; ++i)
            if (g_pf.buf[i].state == kPfReady && g_pf.buf[i].seq < oldest) {
                oldest = g_pf.buf[i].seq;
                pick = i;
            }
        if (pick < 0) {
            ++g_pf.dropped;
            return;
        }
        ++g_pf.stale;
    }
    PfBuffer& b = g_pf.buf[pick];
    b.state = kPfFilling;
    b.src = src;
    b.bytes = bytes;
    b.seq = ++g_pf.seq;
    g_pf.queue.push_back({pick, (const uint8_t*)src, bytes});
    g_pf.cv_work.notify_one();
}

bool sb_pf_take(const void* src, size_t bytes, void* dst, cudaStream_t copy) {
    if (!pf_env_on()) return false;
    int idx = -1;
    bool waited = false;
    const auto t0 = std::chrono::steady_clock::now();
    const auto deadline = t0 + std::chrono::milliseconds(kPfWaitMs);
    {
        std::unique_lock<std::mutex> l(g_pf.mu);
        for (;;) {
            int found = -1;
            for (int i = 0; i < kPfBuffers; ++i) {
                PfBuffer& b = g_pf.buf[i];
                if (b.src != src || b.bytes != bytes) continue;
                if (b.state == kPfFail) {   // the read failed: the miss is staged as usual
                    b.state = kPfFree;
                    b.src = nullptr;
                    return false;
                }
                if (b.state == kPfReady || b.state == kPfFilling) {
                    found = i;
                    break;
                }
            }
            if (found < 0) return false;
            if (g_pf.buf[found].state == kPfReady) {
                g_pf.buf[found].state = kPfTaken;
                idx = found;
                break;
            }
            // still reading: wait for it rather than read the same bytes twice
            waited = true;
            if (g_pf.cv_done.wait_until(l, deadline) == std::cv_status::timeout) {
                ++g_pf.wait_timeouts;
                return false;
            }
        }
        if (waited) {
            ++g_pf.waits;
            g_pf.wait_ns += (unsigned long long)std::chrono::duration_cast<std::chrono::nanoseconds>(
                                std::chrono::steady_clock::now() - t0)
                                .count();
        }
    }
    PfBuffer& b = g_pf.buf[idx];
    bool ok = b.free_ev || cudaEventCreateWithFlags(&b.free_ev, cudaEventDisableTiming) == cudaSuccess;
    ok = ok && sb_cuda_ok(cudaMemcpyAsync(dst, b.mem + b.delta, bytes, cudaMemcpyHostToDevice, copy),
                          "readahead expert H2D") &&
         sb_cuda_ok(cudaEventRecord(b.free_ev, copy), "readahead free record");
    std::lock_guard<std::mutex> l(g_pf.mu);
    b.free_pending = ok;   // the next read into this buffer waits for the copy out
    b.state = kPfFree;
    b.src = nullptr;
    if (ok) {
        ++g_pf.used;
        g_pf.used_bytes += bytes;
    }
    return ok;
}

void sb_stage_stats_get(sb_stage_stats* s) {
    s->staged_bytes = g_st.staged_bytes;
    s->pinned_bytes = g_st.pinned_bytes;
    s->direct_io_reads = g_st.dio_reads;
    s->direct_io_bytes = g_st.dio_bytes;
    s->direct_io_fallbacks = g_st.dio_fallbacks;
    s->waves = g_st.waves;
    std::lock_guard<std::mutex> l(g_pf.mu);
    s->pf_reads = g_pf.reads;
    s->pf_read_bytes = g_pf.read_bytes;
    s->pf_used = g_pf.used;
    s->pf_used_bytes = g_pf.used_bytes;
    s->pf_dropped = g_pf.dropped;
    s->pf_stale = g_pf.stale;
    s->pf_waits = g_pf.waits;
    s->pf_wait_ns = g_pf.wait_ns;
    s->pf_wait_timeouts = g_pf.wait_timeouts;
}

void sb_stage_shutdown() {
    {   // the readahead: readers stopped, buffers released once their copies landed
        {
            std::lock_guard<std::mutex> l(g_pf.mu);
            g_pf.stop = true;
        }
        g_pf.cv_work.notify_all();
        for (std::thread& t : g_pf.readers) t.join();
        std::lock_guard<std::mutex> l(g_pf.mu);
        g_pf.readers.clear();
        g_pf.queue.clear();
        for (PfBuffer& b : g_pf.buf) {
            if (b.free_ev) cudaEventSynchronize(b.free_ev), cudaEventDestroy(b.free_ev);
            if (b.raw) cudaFreeHost(b.raw);
            b = PfBuffer{};
        }
        g_pf.stop = false;
    }
    {
        std::lock_guard<std::mutex> l(g_st.mu);
        g_st.stop = true;
        g_st.cv_work.notify_all();
    }
    for (std::thread& t : g_st.lanes) t.join();
    std::lock_guard<std::mutex> l(g_st.mu);
    g_st.lanes.clear();
    for (int i = 0; i < g_st.depth; ++i) {
        Buffer& b = g_st.buf[i];
        if (b.ev) cudaEventSynchronize(b.ev), cudaEventDestroy(b.ev);
        if (b.raw) cudaFreeHost(b.raw);
        b.ev = nullptr;
        b.raw = b.mem = nullptr;
    }
    g_st.depth = 0;
    g_st.copy = nullptr;
    for (auto& kv : g_st.fds)
        if (kv.second >= 0) ::close(kv.second);
    g_st.fds.clear();
    g_st.maps.clear();
    g_st.maps_loaded = false;
    g_st.queue.clear();
    g_st.pending = 0;
}
