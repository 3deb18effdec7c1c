// libsabah_rt: the C ABI of the routed-expert runtime, for B200 (sm_100a).
//
// Reference interface being replaced: sabah/runtime/cuda/sabah_rt.cu:3039-3903
// (the 42 exported sabah_* symbols). Every entry point keeps the reference's
// signature and error convention: 0 on success, -1 with a message readable
// through sabah_rt_last_error() (one process-wide buffer, last failure wins).
//
// What lives here (host side):
//   * runtime init / streams                       (ref sabah_rt.cu:3190-3232)
//   * the hot-tier slab: one cudaMalloc carved by best fit, coalescing frees
//                                                   (ref :342-424)
//   * the residency table: (source tensor, expert) -> slab range, LRU with
//     per-call completion events guarding reuse    (ref :97-106, 426-800)
//   * miss fill host -> slab on the copy stream    (ref :2051-2116)
//   * router-id download and reuse by ids_key      (ref :3551-3630)
//   * sabah_rt_mul_mat_id_v2, sabah_moe_block and the extensions that run
//     straight from a device-resident expert bank (no id download at all)
//   * counters, snapshot JSON, fp64 self-check, byte verification
// The kernels are in sb_generic.cu and sb_mmid_iq3s.cu.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <list>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <unordered_map>
#include <vector>

#include "sb_kernels.h"
#include "sb_staging.h"
#include "sb_quant.cuh"

#define SABAH_API extern "C" __attribute__((visibility("default")))

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
static char g_err[512] = {0};

void sb_set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

bool sb_cuda_ok(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return true;
    sb_set_error("%s: %s", what, cudaGetErrorString(e));
    return false;
}

// ---------------------------------------------------------------------------
// configuration (environment variables, same names as the reference)
// ---------------------------------------------------------------------------
// "9800000000", "9.8e9", "9.8G", "9800MiB"; a value that does not parse whole
// is refused (ref sabah_rt.cu:276-330 explains the 9.8e9 -> 9 bytes failure).
static bool parse_size(const char* text, size_t& out) {
    if (!text || !*text) return false;
    char* end = nullptr;
    const double v = std::strtod(text, &end);
    if (end == text || !(v > 0)) return false;
    double mul = 1.0;
    if (*end) {
        switch (*end) {
        case 'k': case 'K': mul = 1024.0; break;
        case 'm': case 'M': mul = 1024.0 * 1024; break;
        case 'g': case 'G': mul = 1024.0 * 1024 * 1024; break;
        case 't': case 'T': mul = 1024.0 * 1024 * 1024 * 1024; break;
        default: return false;
        }
        const char* r = end + 1;
        if (*r == 'i' || *r == 'I') ++r;
        if (*r == 'b' || *r == 'B') ++r;
        if (*r) return false;
    }
    const double b = v * mul;
    if (!(b > 0) || b > 1e15) return false;
    out = (size_t)b;
    return true;
}

static size_t hot_bytes_config() {
    const char* env = std::getenv("SABAH_LLAMA_HOT_BYTES");
    if (env && *env) {
        size_t v = 0;
        if (parse_size(env, v)) {
            if (v < ((size_t)256 << 20))
                std::fprintf(stderr, "SABAH_LLAMA: SABAH_LLAMA_HOT_BYTES=%s is only %zu bytes; the hot tier will "
                             "hold almost nothing and most experts will overflow the budget.\n", env, v);
            return v;
        }
        std::fprintf(stderr, "SABAH_LLAMA: cannot read SABAH_LLAMA_HOT_BYTES=%s; using 2 GiB\n", env);
    }
    return (size_t)2 << 30;
}

// ---------------------------------------------------------------------------
// runtime state
// ---------------------------------------------------------------------------
namespace {

struct Runtime {
    int device = -1;
    cudaStream_t copy = nullptr, compute = nullptr;
    int* err_h = nullptr;   // host-mapped pinned word the kernels write
    int* err_d = nullptr;
};
Runtime g_rt;

// -------------------------- slab allocator --------------------------------
struct Slab {
    std::mutex mu;
    char* base = nullptr;
    size_t size = 0;
    std::map<size_t, size_t> free_by_off;           // offset -> bytes
    std::set<std::pair<size_t, size_t>> free_by_len; // (bytes, offset)
    std::unordered_map<void*, size_t> live;          // ptr -> bytes

    void reset_lists() {
        free_by_off.clear();
        free_by_len.clear();
        live.clear();
        if (size) {
            free_by_off[0] = size;
            free_by_len.insert({size, 0});
        }
    }
    bool init_locked(size_t cap) {
        if (base) return true;
        void* p = nullptr;
        if (!sb_cuda_ok(cudaMalloc(&p, cap), "slab allocation")) return false;
        base = (char*)p;
        size = cap;
        reset_lists();
        return true;
    }
    void destroy_locked() {
        if (base) cudaFree(base);
        base = nullptr;
        size = 0;
        reset_lists();
    }
    // best fit: the smallest free range that holds the request, lowest offset on ties
    // sizes are rounded up to 256 B so every range starts 256-byte aligned
    // (the bulk-copy kernels need 16-byte aligned expert bases)
    void* alloc_locked(size_t bytes) {
        if (!base || bytes == 0 || bytes > ((size_t)1 << 60)) return nullptr;
        bytes = (bytes + 255) & ~(size_t)255;
        auto it = free_by_len.lower_bound({bytes, 0});
        if (it == free_by_len.end()) return nullptr;
        const size_t len = it->first, off = it->second;
        free_by_len.erase(it);
        free_by_off.erase(off);
        if (len > bytes) {
            free_by_off[off + bytes] = len - bytes;
            free_by_len.insert({len - bytes, off + bytes});
        }
        void* p = base + off;
        live[p] = bytes;
        return p;
    }
    void free_locked(void* p) {
        auto it = live.find(p);
        if (it == live.end()) return;
        size_t off = (size_t)((char*)p - base), len = it->second;
        live.erase(it);
        auto nx = free_by_off.lower_bound(off);
        if (nx != free_by_off.end() && nx->first == off + len) {   // merge with the next range
            free_by_len.erase({nx->second, nx->first});
            len += nx->second;
            nx = free_by_off.erase(nx);
        }
        if (nx != free_by_off.begin()) {                           // merge with the previous range
            auto pv = std::prev(nx);
            if (pv->first + pv->second == off) {
                free_by_len.erase({pv->second, pv->first});
                off = pv->first;
                len += pv->second;
                free_by_off.erase(pv);
            }
        }
        free_by_off[off] = len;
        free_by_len.insert({len, off});
    }
};
Slab g_slab;

// ---------------------------- residency -----------------------------------
// Residency key: the host tensor's address (the reference's key), the expert,
// its byte size and a tag of the tensor's shape (row stride, rows, k, type),
// so a tensor of another shape met later at a reused address is a miss, not a
// stale hit.
struct Key {
    const void* src;
    int expert;
    size_t bytes;
    uint64_t shape;
    bool operator==(const Key& o) const {
        return src == o.src && expert == o.expert && bytes == o.bytes && shape == o.shape;
    }
};
struct KeyHash {
    size_t operator()(const Key& k) const {
        uint64_t h = (uint64_t)(uintptr_t)k.src * 0x9E3779B97F4A7C15ull;
        h ^= (uint64_t)(uint32_t)k.expert + 0x632BE59BD9B4E019ull + (h << 6) + (h >> 2);
        h ^= (uint64_t)k.bytes * 0xBF58476D1CE4E5B9ull;
        h ^= k.shape * 0x94D049BB133111EBull;
        return (size_t)h;
    }
};
struct Entry {
    void* dev = nullptr;
    size_t bytes = 0;
    uint64_t epoch = 0;      // last call that handed this slot to a kernel
    bool slab = false;       // false: over-budget cudaMalloc
    bool filled = false;
    std::list<Key>::iterator lru;
};

constexpr int kEventRing = 64;   // completion events of the last calls
constexpr uint64_t kIdGroupMax = 4;  // ids reuse window (ref sabah_rt.cu:238)

struct Residency {
    std::mutex mu;
    std::unordered_map<Key, Entry, KeyHash> map;
    std::list<Key> lru;                       // front = most recently used
    size_t capacity = 0, bytes = 0;
    uint64_t epoch = 0;
    cudaEvent_t done[kEventRing] = {};
    uint64_t done_epoch[kEventRing] = {};
    // counters (names as in the reference snapshot)
    uint64_t calls = 0, empty_calls = 0, tokens = 0, hits = 0, misses = 0, evictions = 0;
    uint64_t bytes_fetched = 0, overflow = 0, verify_ok = 0, verify_fail = 0;
    uint64_t id_reuse = 0, id_group_max = 0, device_calls = 0;
    // self-check
    int sc_k = 0;
    double sc_tol = 2e-6, sc_max = 0.0;
    uint64_t sc_ok = 0, sc_fail = 0, sc_multi_token = 0, sc_slot[16] = {};
    std::set<const void*> sc_tensors;
    bool verify = false, verify_all_hits = false;
    uint64_t verify_every = 64;
};
Residency g_res;

struct Fetch {
    const void* src;
    void* dst;
    size_t bytes;
    int expert;
    uint64_t shape;
    const void* src_key;   // the tensor the slot belongs to
};

// ---------------------------- call chain (merged layer fetch) ----------------
// A forward pass issues the same MUL_MAT_ID calls in the same order, and a
// layer's gate, up and down tensors read the same router ids. Each host-source
// call records which tensor followed which, and whether they shared the ids
// (ref sabah_rt.cu:1870-1943, sb_chain_note). With SABAH_LLAMA_LAYER_MERGE=1
// the first call of a layer also reserves and fills its followers' missing
// experts in its own fill wave (ref :1944-2000), so the layer's reads go out
// together and the followers' calls find their experts resident. Off by
// default, as in the reference: the followers' memory must stay mapped, which
// a GGUF mapping does and an arbitrary caller's buffer may not.
struct ChainLink {
    const void* next = nullptr;
    size_t stride = 0;
    uint64_t shape = 0;
    int n_experts = 0;
    bool shares_ids = false;
};
struct Chain {
    std::unordered_map<const void*, ChainLink> links;
    const void* prev = nullptr;
    std::vector<int32_t> prev_ids;
    uint64_t merged_slots = 0;   // follower slots filled in an earlier call's wave
} g_chain;

// the readahead pays only when a call has few ids (ref SB_PF_MAX_TOKENS)
constexpr int kPfMaxTokens = 4;

bool layer_merge_enabled() {
    const char* v = std::getenv("SABAH_LLAMA_LAYER_MERGE");
    return v && (!std::strcmp(v, "1") || !std::strcmp(v, "on"));
}

void residency_reset_locked() {
    g_chain = Chain{};
    for (auto& kv : g_res.map) {
        if (kv.second.slab) {
            std::lock_guard<std::mutex> ls(g_slab.mu);
            g_slab.free_locked(kv.second.dev);
        } else if (kv.second.dev) {
            cudaFree(kv.second.dev);
        }
    }
    g_res.map.clear();
    g_res.lru.clear();
    g_res.bytes = 0;
    g_res.capacity = hot_bytes_config();
    g_res.epoch = 0;
    g_res.calls = g_res.empty_calls = g_res.tokens = g_res.hits = g_res.misses = 0;
    g_res.evictions = g_res.bytes_fetched = g_res.overflow = g_res.verify_ok = g_res.verify_fail = 0;
    g_res.id_reuse = g_res.id_group_max = g_res.device_calls = 0;
    const char* v = std::getenv("SABAH_LLAMA_VERIFY_BYTES");
    g_res.verify = v && (!std::strcmp(v, "1") || !std::strcmp(v, "fetch"));
    g_res.verify_all_hits = v && !std::strcmp(v, "1");
    const char* k = std::getenv("SABAH_LLAMA_SELFCHECK");
    g_res.sc_k = k ? std::atoi(k) : 0;
    const char* tol = std::getenv("SABAH_LLAMA_SELFCHECK_TOL");
    g_res.sc_tol = tol ? std::atof(tol) : 2e-6;
    g_res.sc_ok = g_res.sc_fail = g_res.sc_multi_token = 0;
    g_res.sc_max = 0.0;
    for (auto& c : g_res.sc_slot) c = 0;
    g_res.sc_tensors.clear();
}

// D2H the device copy and compare with the host bytes the slot was filled from
bool verify_slot(const void* dev, const void* host, size_t bytes) {
    std::vector<uint8_t> tmp(bytes);
    if (cudaMemcpy(tmp.data(), dev, bytes, cudaMemcpyDeviceToHost) != cudaSuccess ||
        std::memcmp(tmp.data(), host, bytes) != 0) {
        ++g_res.verify_fail;
        return false;
    }
    ++g_res.verify_ok;
    return true;
}

// Make room for `need` bytes. Entries handed to the call in progress are never
// victims; every other victim's range may still be read by a kernel of the call
// that last used it, so the copy stream is made to wait for that call's
// completion event before anything is written into the range.
void evict_until_locked(size_t need, std::set<uint64_t>& wait_epochs) {
    while (g_res.bytes + need > g_res.capacity) {
        auto it = g_res.lru.end();
        bool found = false;
        while (it != g_res.lru.begin()) {
            --it;
            auto e = g_res.map.find(*it);
            if (e != g_res.map.end() && e->second.epoch != g_res.epoch) {
                found = true;
                break;
            }
        }
        if (!found) return;   // everything resident belongs to this call: exceed the budget
        auto e = g_res.map.find(*it);
        Entry ent = e->second;
        if (ent.epoch + kEventRing > g_res.epoch) wait_epochs.insert(ent.epoch);
        if (ent.slab) {
            std::lock_guard<std::mutex> ls(g_slab.mu);
            g_slab.free_locked(ent.dev);
        } else {
            cudaFree(ent.dev);   // synchronous: no kernel can still be reading it
        }
        g_res.bytes -= ent.bytes;
        g_res.lru.erase(ent.lru);
        g_res.map.erase(e);
        ++g_res.evictions;
    }
}

// Resident device copy of (src_key, expert): a hit, or a reserved slot recorded
// in `miss` for the fill pass. nullptr on failure (message set).
void* slot_locked(const void* src_key, int expert, const void* src, size_t bytes, uint64_t shape,
                  std::vector<Fetch>& miss, std::set<uint64_t>& wait_epochs) {
    const Key key{src_key, expert, bytes, shape};
    auto it = g_res.map.find(key);
    if (it != g_res.map.end()) {
        Entry& e = it->second;
        e.epoch = g_res.epoch;
        g_res.lru.splice(g_res.lru.begin(), g_res.lru, e.lru);
        ++g_res.hits;
        if (e.filled && g_res.verify && (g_res.verify_all_hits || g_res.hits % g_res.verify_every == 0) &&
            !verify_slot(e.dev, src, bytes)) {
            sb_set_error("resident expert %d differs from its source bytes (hit)", expert);
            return nullptr;
        }
        return e.dev;
    }
    ++g_res.misses;
    evict_until_locked(bytes, wait_epochs);
    void* dev = nullptr;
    bool from_slab = false;
    {
        std::lock_guard<std::mutex> ls(g_slab.mu);
        if (!g_slab.base) g_slab.init_locked(hot_bytes_config());
        if (g_res.bytes + bytes <= g_res.capacity) dev = g_slab.alloc_locked(bytes);
        from_slab = dev != nullptr;
    }
    if (!dev) {
        // documented behaviour: exceed the budget with a plain allocation rather
        // than fail the call (ref sabah_rt.cu:725-735); counted as overflow
        ++g_res.overflow;
        if (!sb_cuda_ok(cudaMalloc(&dev, bytes), "over-budget expert allocation")) return nullptr;
    }
    g_res.lru.push_front(key);
    Entry e;
    e.dev = dev;
    e.bytes = bytes;
    e.epoch = g_res.epoch;
    e.slab = from_slab;
    e.filled = false;
    e.lru = g_res.lru.begin();
    g_res.map.emplace(key, e);
    g_res.bytes += bytes;
    g_res.bytes_fetched += bytes;
    miss.push_back({src, dev, bytes, expert, shape, src_key});
    return dev;
}

// Copy every reserved slot in from the host on the copy stream.
bool fill_locked(const std::vector<Fetch>& miss, const std::set<uint64_t>& wait_epochs) {
    for (uint64_t ep : wait_epochs) {
        const int r = (int)(ep % kEventRing);
        if (g_res.done[r] && g_res.done_epoch[r] == ep &&
            !sb_cuda_ok(cudaStreamWaitEvent(g_rt.copy, g_res.done[r], 0), "copy stream wait"))
            return false;
    }
    // bytes a readahead already holds (or is reading) are copied from its
    // buffer; pinned sources by direct DMA; pageable or file-mapped ones through
    // the pinned staging ring and its reader lanes (sb_staging.cu)
    std::vector<sb_fill> fills;
    fills.reserve(miss.size());
    const bool pf = sb_pf_enabled();
    for (const Fetch& f : miss)
        if (!(pf && sb_pf_take(f.src, f.bytes, f.dst, g_rt.copy))) fills.push_back({f.dst, f.src, f.bytes});
    if (!fills.empty() && !sb_stage_fill(fills.data(), (int)fills.size(), g_rt.copy)) return false;
    for (const Fetch& f : miss) {
        auto it = g_res.map.find(Key{f.src_key, f.expert, f.bytes, f.shape});
        if (it != g_res.map.end()) it->second.filled = true;
        if (g_res.verify) {
            if (!sb_cuda_ok(cudaStreamSynchronize(g_rt.copy), "verify sync")) return false;
            if (!verify_slot(f.dst, f.src, f.bytes)) {
                sb_set_error("fetched expert %d differs from its source bytes (miss)", f.expert);
                return false;
            }
        }
    }
    return true;
}

// completion event of the call in progress, recorded after its kernel
bool record_done_locked(cudaStream_t st) {
    const int r = (int)(g_res.epoch % kEventRing);
    if (!g_res.done[r]) {
        if (!sb_cuda_ok(cudaEventCreateWithFlags(&g_res.done[r], cudaEventDisableTiming), "event create"))
            return false;
    } else if (g_res.done_epoch[r] + kEventRing == g_res.epoch) {
        // reusing the slot of a call kEventRing calls ago: make sure it is finished,
        // so any entry older than the ring is known to be free of readers
        cudaEventSynchronize(g_res.done[r]);
    }
    g_res.done_epoch[r] = g_res.epoch;
    return sb_cuda_ok(cudaEventRecord(g_res.done[r], st), "event record");
}

// ------------------------- scratch / staging -------------------------------
struct Scratch {
    void** ptr_table = nullptr;
    size_t ptr_cap = 0;
    cudaEvent_t ready = nullptr;
    int32_t* ids_h = nullptr;     // pinned id download buffer
    size_t ids_cap = 0;
};
Scratch g_scr;

bool ptr_table(size_t bytes, void*** out) {
    if (bytes > g_scr.ptr_cap) {
        if (g_scr.ptr_table) cudaFree(g_scr.ptr_table);
        g_scr.ptr_table = nullptr;
        g_scr.ptr_cap = 0;
        const size_t cap = std::max<size_t>(bytes, 1 << 16);
        if (!sb_cuda_ok(cudaMalloc(&g_scr.ptr_table, cap), "pointer table allocation")) return false;
        g_scr.ptr_cap = cap;
    }
    *out = g_scr.ptr_table;
    return true;
}

bool ids_buffer(size_t bytes) {
    if (bytes <= g_scr.ids_cap) return true;
    if (g_scr.ids_h) cudaFreeHost(g_scr.ids_h);
    g_scr.ids_h = nullptr;
    g_scr.ids_cap = 0;
    const size_t cap = std::max<size_t>(bytes, 1 << 16);
    if (!sb_cuda_ok(cudaHostAlloc((void**)&g_scr.ids_h, cap, cudaHostAllocDefault), "id buffer")) return false;
    g_scr.ids_cap = cap;
    return true;
}

void scratch_destroy() {
    if (g_scr.ptr_table) cudaFree(g_scr.ptr_table);
    if (g_scr.ready) cudaEventDestroy(g_scr.ready);
    if (g_scr.ids_h) cudaFreeHost(g_scr.ids_h);
    g_scr = Scratch{};
}

// ---------------------------- pinned pool ----------------------------------
struct PinnedBlock {
    void* ptr;
    size_t bytes;
    int refs;
};
std::mutex g_pin_mu;
std::vector<PinnedBlock> g_pinned;

void pinned_destroy() {
    std::lock_guard<std::mutex> l(g_pin_mu);
    for (auto& b : g_pinned) cudaFreeHost(b.ptr);
    g_pinned.clear();
}

// ----------------------- device source detection ---------------------------
// The extension of the v2 contract: a `source` in device memory is a resident
// bank and is read in place.
bool is_device_pointer(const void* p) {
    static const void* last = nullptr;
    static bool last_dev = false;
    if (p == last) return last_dev;
    cudaPointerAttributes at{};
    bool dev = false;
    if (cudaPointerGetAttributes(&at, p) == cudaSuccess)
        dev = at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
    cudaGetLastError();   // a plain host pointer may leave an error behind on old drivers
    last = p;
    last_dev = dev;
    return dev;
}

bool device_errors_clear() {
    if (g_rt.err_h && *(volatile int*)g_rt.err_h != SB_DERR_NONE) {
        const int code = *(volatile int*)g_rt.err_h;
        *(volatile int*)g_rt.err_h = SB_DERR_NONE;
        sb_block_scratch_invalidate();
        sb_decode_scratch_invalidate();
        sb_set_error("%s (device error %d, reported by the first call after the kernel ran)",
                     code == SB_DERR_BAD_ID ? "a kernel found an expert id outside [0, n_experts)"
                     : code == SB_DERR_MISALIGNED ? "an expert base was not 16-byte aligned"
                     : "a kernel gave up waiting for its weight tiles", code);
        return false;
    }
    return true;
}

uint64_t mix64(uint64_t z) {   // splitmix64 finaliser, for self-check sampling
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

bool host_dequant(const uint8_t* src, float* dst, int qt, long long n) {
    const int be = sb_block_elems(qt);
    if (be == 0 || n % be) return false;
    const long long nsub = n / 32;
    auto l = [&](auto tag) {
        for (long long i = 0; i < nsub; ++i) sb_dequant32<decltype(tag)::value>(src, (int)i, dst + 32 * i);
    };
    return sb_dispatch_qt(qt, l);
}

// fp64 recomputation of K sampled (token, slot) outputs of the call that just
// ran (the reference's SABAH_LLAMA_SELFCHECK, sabah_rt.cu:3435-3492).
void selfcheck(const void* source, bool source_on_device, const sb_mmid_args& a, const int32_t* ids_host,
               size_t ids_id_stride, size_t ids_token_stride, size_t expert_stride, cudaStream_t st, uint64_t call_no) {
    if (g_res.sc_k <= 0) return;
    cudaStreamSynchronize(st);
    const int pairs = a.n_ids * a.n_tokens;
    const int samples = std::min(g_res.sc_k, pairs);
    std::vector<float> x(a.k), out(a.rows), w(a.k);
    std::vector<uint8_t> rowbuf(a.row_stride);
    const uint64_t h0 = mix64(call_no * 0x100000001B3ull + 0x5AB4ull);
    for (int s = 0; s < samples; ++s) {
        int t, slot;
        if (g_res.sc_k >= pairs) {       // every pair exactly once
            t = s / a.n_ids;
            slot = s % a.n_ids;
        } else {
            const uint64_t h = mix64(h0 + (uint64_t)s);
            t = (int)(h % (uint64_t)a.n_tokens);
            slot = (int)((mix64(h) + (uint64_t)s) % (uint64_t)a.n_ids);
        }
        const int expert = *(const int32_t*)((const uint8_t*)ids_host + (size_t)t * ids_token_stride +
                                             (size_t)slot * ids_id_stride);
        const uint8_t* xp = (const uint8_t*)a.x + (size_t)(slot % a.x_rows) * a.x_id_stride + (size_t)t * a.x_token_stride;
        const uint8_t* op = (const uint8_t*)a.dst + (size_t)t * a.dst_token_stride + (size_t)slot * a.dst_id_stride;
        if (cudaMemcpy(x.data(), xp, (size_t)a.k * 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
            cudaMemcpy(out.data(), op, (size_t)a.rows * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
            ++g_res.sc_fail;
            continue;
        }
        const uint8_t* wexp = (const uint8_t*)source + (size_t)expert * expert_stride;
        double num = 0.0, den = 0.0;
        for (int r = 0; r < a.rows; ++r) {
            const uint8_t* rp = wexp + (size_t)r * a.row_stride;
            if (source_on_device) {
                cudaMemcpy(rowbuf.data(), rp, a.row_stride, cudaMemcpyDeviceToHost);
                rp = rowbuf.data();
            }
            host_dequant(rp, w.data(), a.qt, a.k);
            double acc = 0.0;
            for (int c = 0; c < a.k; ++c) acc += (double)w[c] * (double)x[c];
            const double e = (double)out[r] - acc;
            num += e * e;
            den += acc * acc;
        }
        const double rel = den > 0 ? std::sqrt(num / den) : std::sqrt(num);
        if (rel <= g_res.sc_tol) {
            ++g_res.sc_ok;
        } else {
            if (g_res.sc_fail == 0)
                std::fprintf(stderr, "SABAH_SELFCHECK_FAIL call=%llu token=%d/%d slot=%d expert=%d rel_l2=%.3e\n",
                             (unsigned long long)call_no, t, a.n_tokens, slot, expert, rel);
            ++g_res.sc_fail;
        }
        g_res.sc_max = std::max(g_res.sc_max, rel);
        if (slot < 16) ++g_res.sc_slot[slot];
        if (a.n_tokens > 1) ++g_res.sc_multi_token;
        g_res.sc_tensors.insert(source);
    }
}

int snapshot_json(char* buf, size_t n) {
    std::lock_guard<std::mutex> l(g_res.mu);
    sb_stage_stats ss{};
    sb_stage_stats_get(&ss);
    char slots[256];
    int o = 0;
    for (int i = 0; i < 16; ++i)
        o += std::snprintf(slots + o, sizeof(slots) - o, "%s%llu", i ? "," : "", (unsigned long long)g_res.sc_slot[i]);
    return std::snprintf(
        buf, n,
        "{\"calls\":%llu,\"empty_calls\":%llu,\"tokens\":%llu,\"lookups\":%llu,\"hits\":%llu,"
        "\"misses\":%llu,\"evictions\":%llu,\"bytes_fetched\":%llu,\"resident_bytes\":%llu,"
        "\"overflow\":%llu,\"verify_ok\":%llu,\"verify_fail\":%llu,"
        "\"selfcheck_k\":%d,\"selfcheck_ok\":%llu,\"selfcheck_fail\":%llu,\"selfcheck_max_rel_l2\":%.6e,"
        "\"selfcheck_multi_token\":%llu,\"selfcheck_tensors\":%llu,\"selfcheck_slots\":[%s],"
        "\"sentinel\":%d,\"device_calls\":%llu,\"id_reuse\":%llu,"
        "\"staged_bytes\":%llu,\"pinned_fill_bytes\":%llu,\"direct_io_reads\":%llu,\"direct_io_bytes\":%llu,"
        "\"direct_io_fallbacks\":%llu,\"fill_waves\":%llu,\"merged_slots\":%llu,"
        "\"prefetch_enabled\":%d,\"prefetch_reads\":%llu,\"prefetch_read_bytes\":%llu,\"prefetch_used\":%llu,"
        "\"prefetch_used_bytes\":%llu,\"prefetch_dropped\":%llu,\"prefetch_stale\":%llu,\"prefetch_waits\":%llu,"
        "\"prefetch_wait_ms\":%.3f,\"prefetch_wait_timeouts\":%llu}",
        (unsigned long long)g_res.calls, (unsigned long long)g_res.empty_calls, (unsigned long long)g_res.tokens,
        (unsigned long long)(g_res.hits + g_res.misses), (unsigned long long)g_res.hits,
        (unsigned long long)g_res.misses, (unsigned long long)g_res.evictions,
        (unsigned long long)g_res.bytes_fetched, (unsigned long long)g_res.bytes,
        (unsigned long long)g_res.overflow, (unsigned long long)g_res.verify_ok,
        (unsigned long long)g_res.verify_fail, g_res.sc_k, (unsigned long long)g_res.sc_ok,
        (unsigned long long)g_res.sc_fail, g_res.sc_max, (unsigned long long)g_res.sc_multi_token,
        (unsigned long long)g_res.sc_tensors.size(), slots, SABAH_SENTINEL,
        (unsigned long long)g_res.device_calls, (unsigned long long)g_res.id_reuse, ss.staged_bytes, ss.pinned_bytes,
        ss.direct_io_reads, ss.direct_io_bytes, ss.direct_io_fallbacks, ss.waves,
        (unsigned long long)g_chain.merged_slots, sb_pf_enabled() ? 1 : 0, ss.pf_reads, ss.pf_read_bytes, ss.pf_used,
        ss.pf_used_bytes, ss.pf_dropped, ss.pf_stale, ss.pf_waits, (double)ss.pf_wait_ns / 1e6, ss.pf_wait_timeouts);
}

void status_write() {
    static const char* path = std::getenv("SABAH_LLAMA_STATUS_FILE");
    if (!path || !*path) return;
    char buf[2048];
    snapshot_json(buf, sizeof(buf));
    if (FILE* f = std::fopen(path, "wb")) {
        std::fputs(buf, f);
        std::fputc('\n', f);
        std::fclose(f);
    }
}

void report_at_exit() {
    if (!std::getenv("SABAH_LLAMA_TRACE")) return;
    char buf[2048];
    snapshot_json(buf, sizeof(buf));
    std::fprintf(stderr, "SABAH_DIAG calls=%llu tokens=%llu lookups=%llu overflow=%llu verify_ok=%llu verify_fail=%llu\n",
                 (unsigned long long)g_res.calls, (unsigned long long)g_res.tokens,
                 (unsigned long long)(g_res.hits + g_res.misses), (unsigned long long)g_res.overflow,
                 (unsigned long long)g_res.verify_ok, (unsigned long long)g_res.verify_fail);
    std::fprintf(stderr, "SABAH_SNAPSHOT %s\n", buf);
}

bool ensure_init() {
    if (g_rt.copy) return true;
    sb_set_error("sabah_rt_init has not been called");
    return false;
}

// ---------------------- Linux file resolution probes ----------------------
struct DiskFile {
    std::string path;
    int fd = -1;
    uint64_t size = 0;
};
std::mutex g_disk_mu;
std::vector<DiskFile> g_disk;

// ptr -> (file, offset) through /proc/self/maps (the Linux counterpart of the
// reference's VirtualQuery + GetMappedFileName, sabah_rt.cu:952-1031)
bool resolve_ptr(const void* ptr, std::string& path, uint64_t& off, std::string& why) {
    FILE* f = std::fopen("/proc/self/maps", "r");
    if (!f) {
        why = "no /proc/self/maps";
        return false;
    }
    char line[4096];
    const uintptr_t p = (uintptr_t)ptr;
    bool ok = false;
    while (std::fgets(line, sizeof(line), f)) {
        unsigned long lo, hi, foff;
        char perms[8], dev[16];
        unsigned long inode;
        int consumed = 0;
        if (std::sscanf(line, "%lx-%lx %7s %lx %15s %lu %n", &lo, &hi, perms, &foff, dev, &inode, &consumed) < 6) continue;
        if (p < lo || p >= hi) continue;
        std::string rest = consumed > 0 ? std::string(line + consumed) : std::string();
        while (!rest.empty() && (rest.back() == '\n' || rest.back() == ' ')) rest.pop_back();
        if (inode == 0 || rest.empty() || rest[0] != '/') {
            why = "pointer is not in a file mapping";
        } else {
            path = rest;
            off = (uint64_t)(p - lo) + foff;
            ok = true;
        }
        break;
    }
    std::fclose(f);
    if (!ok && why.empty()) why = "pointer not mapped";
    return ok;
}

}  // namespace

// ===========================================================================
// C API
// ===========================================================================
SABAH_API const char* sabah_rt_last_error(void) { return g_err; }

SABAH_API int sabah_rt_init(int device) {
    if (!sb_cuda_ok(cudaSetDevice(device), "cudaSetDevice")) return -1;
    if (!g_rt.copy) {
        // blocking streams, as the reference creates them: work a caller queued
        // on the legacy default stream is ordered before anything issued here
        SB_CUDA(cudaStreamCreate(&g_rt.copy), "create copy stream");
        SB_CUDA(cudaStreamCreate(&g_rt.compute), "create compute stream");
    }
    if (!g_rt.err_h) {
        SB_CUDA(cudaHostAlloc((void**)&g_rt.err_h, sizeof(int), cudaHostAllocMapped), "error word");
        *g_rt.err_h = SB_DERR_NONE;
        SB_CUDA(cudaHostGetDevicePointer((void**)&g_rt.err_d, g_rt.err_h, 0), "error word mapping");
    }
    g_rt.device = device;
    {
        std::lock_guard<std::mutex> l(g_res.mu);
        residency_reset_locked();
    }
    {
        std::lock_guard<std::mutex> l(g_slab.mu);
        if (!g_slab.init_locked(hot_bytes_config())) return -1;
    }
    static bool registered = false;
    if (!registered) {
        std::atexit(report_at_exit);
        registered = true;
    }
    return 0;
}

SABAH_API int sabah_rt_shutdown(void) {
    if (g_rt.copy) {
        cudaStreamSynchronize(g_rt.copy);
        cudaStreamSynchronize(g_rt.compute);
    }
    {
        std::lock_guard<std::mutex> l(g_res.mu);
        residency_reset_locked();
        for (auto& e : g_res.done)
            if (e) cudaEventDestroy(e), e = nullptr;
    }
    {
        std::lock_guard<std::mutex> l(g_slab.mu);
        g_slab.destroy_locked();
    }
    sb_stage_shutdown();
    scratch_destroy();
    pinned_destroy();
    if (g_rt.copy) cudaStreamDestroy(g_rt.copy);
    if (g_rt.compute) cudaStreamDestroy(g_rt.compute);
    g_rt.copy = g_rt.compute = nullptr;
    if (g_rt.err_h) cudaFreeHost(g_rt.err_h);
    g_rt.err_h = g_rt.err_d = nullptr;
    return 0;
}

SABAH_API int sabah_rt_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

SABAH_API void* sabah_dev_alloc(size_t bytes) {
    void* p = nullptr;
    if (!sb_cuda_ok(cudaMalloc(&p, bytes), "cudaMalloc")) return nullptr;
    return p;
}
SABAH_API void sabah_dev_free(void* p) {
    if (p) cudaFree(p);
}

// pinned host blocks are pooled and reused; released at shutdown
SABAH_API void* sabah_host_alloc(size_t bytes) {
    std::lock_guard<std::mutex> l(g_pin_mu);
    for (auto& b : g_pinned)
        if (b.refs == 0 && b.bytes >= bytes) {
            b.refs = 1;
            return b.ptr;
        }
    void* p = nullptr;
    if (!sb_cuda_ok(cudaHostAlloc(&p, bytes, cudaHostAllocDefault), "cudaHostAlloc")) return nullptr;
    g_pinned.push_back({p, bytes, 1});
    return p;
}
SABAH_API void sabah_host_free(void* p) {
    if (!p) return;
    std::lock_guard<std::mutex> l(g_pin_mu);
    for (auto& b : g_pinned)
        if (b.ptr == p) {
            if (b.refs > 0) --b.refs;
            return;
        }
    cudaFreeHost(p);
}
SABAH_API int sabah_host_register(void* ptr, size_t bytes) {
    return sb_cuda_ok(cudaHostRegister(ptr, bytes, cudaHostRegisterDefault), "cudaHostRegister") ? 0 : -1;
}
SABAH_API int sabah_host_unregister(void* ptr) {
    return sb_cuda_ok(cudaHostUnregister(ptr), "cudaHostUnregister") ? 0 : -1;
}
SABAH_API int sabah_dev_mem(size_t* freeb, size_t* totalb) {
    return sb_cuda_ok(cudaMemGetInfo(freeb, totalb), "cudaMemGetInfo") ? 0 : -1;
}
SABAH_API int sabah_memcpy_h2d(void* dst, const void* src, size_t n) {
    return sb_cuda_ok(cudaMemcpy(dst, src, n, cudaMemcpyHostToDevice), "memcpy h2d") ? 0 : -1;
}
SABAH_API int sabah_memcpy_d2h(void* dst, const void* src, size_t n) {
    return sb_cuda_ok(cudaMemcpy(dst, src, n, cudaMemcpyDeviceToHost), "memcpy d2h") ? 0 : -1;
}
SABAH_API int sabah_memset_d(void* dst, int v, size_t n) {
    return sb_cuda_ok(cudaMemset(dst, v, n), "memset") ? 0 : -1;
}
SABAH_API int sabah_h2d_async(void* dst, const void* src, size_t n) {
    if (!ensure_init()) return -1;
    return sb_cuda_ok(cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, g_rt.copy), "memcpyAsync h2d") ? 0 : -1;
}

SABAH_API void* sabah_event_create(void) {
    cudaEvent_t ev;
    if (!sb_cuda_ok(cudaEventCreate(&ev), "eventCreate")) return nullptr;
    return (void*)ev;
}
SABAH_API void sabah_event_destroy(void* ev) {
    if (ev) cudaEventDestroy((cudaEvent_t)ev);
}
SABAH_API int sabah_event_record_copy(void* ev) {
    if (!ensure_init()) return -1;
    return sb_cuda_ok(cudaEventRecord((cudaEvent_t)ev, g_rt.copy), "record copy") ? 0 : -1;
}
SABAH_API int sabah_event_record_compute(void* ev) {
    if (!ensure_init()) return -1;
    return sb_cuda_ok(cudaEventRecord((cudaEvent_t)ev, g_rt.compute), "record compute") ? 0 : -1;
}
SABAH_API int sabah_compute_wait_event(void* ev) {
    if (!ensure_init()) return -1;
    return sb_cuda_ok(cudaStreamWaitEvent(g_rt.compute, (cudaEvent_t)ev, 0), "streamWaitEvent") ? 0 : -1;
}
// the copy stream waits for a compute event: a slot about to be overwritten may
// still be read by a submitted kernel
SABAH_API int sabah_copy_wait_event(void* ev) {
    if (!ensure_init()) return -1;
    return sb_cuda_ok(cudaStreamWaitEvent(g_rt.copy, (cudaEvent_t)ev, 0), "copyStreamWaitEvent") ? 0 : -1;
}
SABAH_API float sabah_event_elapsed_ms(void* a, void* b) {
    float ms = -1.f;
    cudaEventSynchronize((cudaEvent_t)b);
    if (!sb_cuda_ok(cudaEventElapsedTime(&ms, (cudaEvent_t)a, (cudaEvent_t)b), "elapsed")) return -1.f;
    return ms;
}
SABAH_API int sabah_event_sync(void* ev) {
    return sb_cuda_ok(cudaEventSynchronize((cudaEvent_t)ev), "eventSynchronize") ? 0 : -1;
}
SABAH_API int sabah_event_query(void* ev) {
    const cudaError_t e = cudaEventQuery((cudaEvent_t)ev);
    if (e == cudaSuccess) return 1;
    if (e == cudaErrorNotReady) {
        cudaGetLastError();
        return 0;
    }
    sb_cuda_ok(e, "eventQuery");
    return -1;
}
SABAH_API int sabah_sync_copy(void) {
    if (!ensure_init()) return -1;
    return sb_cuda_ok(cudaStreamSynchronize(g_rt.copy), "sync copy") ? 0 : -1;
}
SABAH_API int sabah_sync_compute(void) {
    if (!ensure_init()) return -1;
    return sb_cuda_ok(cudaStreamSynchronize(g_rt.compute), "sync compute") ? 0 : -1;
}
SABAH_API int sabah_sync_all(void) {
    return sb_cuda_ok(cudaDeviceSynchronize(), "sync device") ? 0 : -1;
}

// Reference fused block ABI (sabah_rt.cu:3362-3378): one token; d_ptrs is a
// device array [gate x n_used, up x n_used, down x n_used]; d_w the routing
// weights; d_h scratch of n_used * ff floats. Runs on the runtime's compute stream.
SABAH_API int sabah_moe_block(const float* d_x, float* d_out, float* d_h, const void* const* d_ptrs, const float* d_w,
                              int d_model, int ff, int n_used, int qt_gate, int qt_up, int qt_down, int accumulate) {
    if (!ensure_init()) return -1;
    if ((d_model % 32) || (ff % 32)) {
        sb_set_error("d_model and ff must be multiples of 32");
        return -1;
    }
    if (!sb_row_bytes_of(qt_gate, d_model) || !sb_row_bytes_of(qt_up, d_model) || !sb_row_bytes_of(qt_down, ff)) {
        sb_set_error("unsupported quant type or row length for the block (%d/%d/%d)", qt_gate, qt_up, qt_down);
        return -1;
    }
    if (n_used <= 0) return 0;
    sb_block_args a{};
    a.gate.ptrs = d_ptrs;
    a.up.ptrs = d_ptrs + n_used;
    a.down.ptrs = d_ptrs + 2 * n_used;
    a.x = d_x;
    a.h = d_h;
    a.out = d_out;
    a.w = d_w;
    a.d_model = d_model;
    a.ff = ff;
    a.n_used = n_used;
    a.n_tokens = 1;
    a.qt_gate = qt_gate;
    a.qt_up = qt_up;
    a.qt_down = qt_down;
    a.accumulate = accumulate;
    a.err = g_rt.err_d;
    return sb_launch_block(a, g_rt.compute);
}

// Extension: the fused block straight from device-resident banks, n_tokens
// tokens, routing ids read on the device (no host round trip, no pointer
// table). Banks are [n_experts][rows][row bytes]; ids/w [n_tokens][n_used];
// x/out [n_tokens][d_model]; h scratch [n_tokens][n_used][ff]. stream NULL ->
// the runtime's compute stream.
SABAH_API int sabah_moe_block_ids(const void* gate_bank, const void* up_bank, const void* down_bank,
                                  size_t gu_expert_stride, size_t down_expert_stride, int n_experts,
                                  const int32_t* d_ids, const float* d_w, const float* d_x, float* d_out, float* d_h,
                                  int d_model, int ff, int n_used, int n_tokens, int qt_gate, int qt_up, int qt_down,
                                  int accumulate, void* stream) {
    if (!ensure_init()) return -1;
    if (!device_errors_clear()) return -1;
    if (!gate_bank || !up_bank || !down_bank || !d_ids || !d_w || !d_x || !d_out || !d_h) {
        sb_set_error("invalid moe_block_ids arguments");
        return -1;
    }
    if ((d_model % 32) || (ff % 32) || n_used <= 0 || n_tokens < 0 || n_experts <= 0) {
        sb_set_error("invalid moe_block_ids geometry");
        return -1;
    }
    if (!sb_row_bytes_of(qt_gate, d_model) || !sb_row_bytes_of(qt_up, d_model) || !sb_row_bytes_of(qt_down, ff)) {
        sb_set_error("unsupported quant type or row length for the block (%d/%d/%d)", qt_gate, qt_up, qt_down);
        return -1;
    }
    if (n_tokens == 0) return 0;
    sb_block_args a{};
    auto bank = [&](const void* b, size_t stride) {
        sb_experts e{};
        e.base = (const uint8_t*)b;
        e.expert_stride = stride;
        e.ids = d_ids;
        e.ids_id_stride = 4;
        e.ids_token_stride = (size_t)4 * n_used;
        e.n_experts = n_experts;
        return e;
    };
    a.gate = bank(gate_bank, gu_expert_stride);
    a.up = bank(up_bank, gu_expert_stride);
    a.down = bank(down_bank, down_expert_stride);
    a.x = d_x;
    a.h = d_h;
    a.out = d_out;
    a.w = d_w;
    a.d_model = d_model;
    a.ff = ff;
    a.n_used = n_used;
    a.n_tokens = n_tokens;
    a.qt_gate = qt_gate;
    a.qt_up = qt_up;
    a.qt_down = qt_down;
    a.accumulate = accumulate;
    a.err = g_rt.err_d;
    return sb_launch_block(a, stream ? (cudaStream_t)stream : g_rt.compute);
}

// sabah_moe_block_ids over gathered inputs: token t's input is row d_xrows[t]
// of d_x (n_xrows rows). No reference counterpart: the expert-parallel bank
// calls it with the all-gathered activations and the rows of its local
// (token, slot) pairs. IQ3_S blocks that take the one-launch path read the
// rows in place; every other case gathers them into scratch first. A row index
// outside [0, n_xrows) gives NaN outputs and the device error.
SABAH_API int sabah_moe_block_gather(const void* gate_bank, const void* up_bank, const void* down_bank,
                                     size_t gu_expert_stride, size_t down_expert_stride, int n_experts,
                                     const int32_t* d_ids, const float* d_w, const float* d_x, const int32_t* d_xrows,
                                     int n_xrows, float* d_out, float* d_h, int d_model, int ff, int n_used,
                                     int n_tokens, int qt_gate, int qt_up, int qt_down, int accumulate, void* stream) {
    if (!ensure_init()) return -1;
    if (!device_errors_clear()) return -1;
    if (!gate_bank || !up_bank || !down_bank || !d_ids || !d_w || !d_x || !d_xrows || !d_out || !d_h ||
        n_xrows <= 0) {
        sb_set_error("invalid moe_block_gather arguments");
        return -1;
    }
    if ((d_model % 32) || (ff % 32) || n_used <= 0 || n_tokens < 0 || n_experts <= 0) {
        sb_set_error("invalid moe_block_gather geometry");
        return -1;
    }
    if (!sb_row_bytes_of(qt_gate, d_model) || !sb_row_bytes_of(qt_up, d_model) || !sb_row_bytes_of(qt_down, ff)) {
        sb_set_error("unsupported quant type or row length for the block (%d/%d/%d)", qt_gate, qt_up, qt_down);
        return -1;
    }
    if (n_tokens == 0) return 0;
    const cudaStream_t st = stream ? (cudaStream_t)stream : g_rt.compute;
    sb_block_args a{};
    auto bank = [&](const void* b, size_t stride) {
        sb_experts e{};
        e.base = (const uint8_t*)b;
        e.expert_stride = stride;
        e.ids = d_ids;
        e.ids_id_stride = 4;
        e.ids_token_stride = (size_t)4 * n_used;
        e.n_experts = n_experts;
        return e;
    };
    a.gate = bank(gate_bank, gu_expert_stride);
    a.up = bank(up_bank, gu_expert_stride);
    a.down = bank(down_bank, down_expert_stride);
    a.x = d_x;
    a.xrows = d_xrows;
    a.n_xrows = n_xrows;
    a.h = d_h;
    a.out = d_out;
    a.w = d_w;
    a.d_model = d_model;
    a.ff = ff;
    a.n_used = n_used;
    a.n_tokens = n_tokens;
    a.qt_gate = qt_gate;
    a.qt_up = qt_up;
    a.qt_down = qt_down;
    a.accumulate = accumulate;
    a.err = g_rt.err_d;
    if (qt_gate == SB_IQ3_S && qt_up == SB_IQ3_S && qt_down == SB_IQ3_S) {
        const int taken = sb_try_block_iq3s(a, st);
        if (taken != 0) return taken > 0 ? 0 : -1;
    }
    // gather the rows into scratch (grown on demand), then the plain block
    static float* rows = nullptr;
    static size_t cap = 0;
    const size_t need = (size_t)n_tokens * d_model;
    if (need > cap) {
        if (rows) {
            cudaDeviceSynchronize();   // no kernel of an earlier call may still use it
            cudaFree(rows);
            rows = nullptr;
            cap = 0;
        }
        if (!sb_cuda_ok(cudaMalloc(&rows, need * sizeof(float)), "block gather scratch")) return -1;
        cap = need;
    }
    if (sb_gather_rows(d_x, n_xrows, d_xrows, n_tokens, d_model, rows, g_rt.err_d, st) != 0) return -1;
    a.x = rows;
    a.xrows = nullptr;
    a.n_xrows = 0;
    return sb_launch_block(a, st);
}

// sabah_moe_block_ids over the fixed scratch of the IQ3_S kernels: no device or
// host memory is allocated, at the price of a size limit and of calls that
// must not overlap on the GPU (they share that scratch).
SABAH_API int sabah_moe_block_ids_noalloc(const void* gate_bank, const void* up_bank, const void* down_bank,
                                          size_t gu_expert_stride, size_t down_expert_stride, int n_experts,
                                          const int32_t* d_ids, const float* d_w, const float* d_x, float* d_out,
                                          float* d_h, int d_model, int ff, int n_used, int n_tokens, int qt_gate,
                                          int qt_up, int qt_down, int accumulate, void* stream) {
    if (!ensure_init()) return -1;
    if (!device_errors_clear()) return -1;
    if (!gate_bank || !up_bank || !down_bank || !d_ids || !d_w || !d_x || !d_out || !d_h) {
        sb_set_error("invalid moe_block_ids_noalloc arguments");
        return -1;
    }
    if ((d_model % 32) || (ff % 32) || n_used <= 0 || n_tokens < 0 || n_experts <= 0) {
        sb_set_error("invalid moe_block_ids_noalloc geometry");
        return -1;
    }
    if (n_tokens == 0) return 0;
    sb_block_args a{};
    auto bank = [&](const void* b, size_t stride) {
        sb_experts e{};
        e.base = (const uint8_t*)b;
        e.expert_stride = stride;
        e.ids = d_ids;
        e.ids_id_stride = 4;
        e.ids_token_stride = (size_t)4 * n_used;
        e.n_experts = n_experts;
        return e;
    };
    a.gate = bank(gate_bank, gu_expert_stride);
    a.up = bank(up_bank, gu_expert_stride);
    a.down = bank(down_bank, down_expert_stride);
    a.x = d_x;
    a.h = d_h;
    a.out = d_out;
    a.w = d_w;
    a.d_model = d_model;
    a.ff = ff;
    a.n_used = n_used;
    a.n_tokens = n_tokens;
    a.qt_gate = qt_gate;
    a.qt_up = qt_up;
    a.qt_down = qt_down;
    a.accumulate = accumulate;
    a.err = g_rt.err_d;
    return sb_block_iq3s_fixed(a, stream ? (cudaStream_t)stream : g_rt.compute);
}

// Reads and clears the device error word (1 = an out-of-range expert id met
// by a kernel reading a device-resident bank). Returns the code, 0 if none.
SABAH_API int sabah_rt_device_error(void) {
    if (!g_rt.err_h) return 0;
    const int c = *(volatile int*)g_rt.err_h;
    *(volatile int*)g_rt.err_h = SB_DERR_NONE;
    if (c != SB_DERR_NONE) {
        sb_block_scratch_invalidate();
        sb_decode_scratch_invalidate();
    }
    return c;
}

SABAH_API int sabah_rt_mul_mat_id_v2(const void* source, size_t expert_stride, size_t row_stride, const void* d_x,
                                     size_t x_id_stride, int x_rows, size_t x_token_stride, const void* d_ids,
                                     size_t ids_id_stride, size_t ids_token_stride, int n_ids, int n_tokens,
                                     float* d_dst, size_t dst_id_stride, size_t dst_token_stride, int rows, int k,
                                     int n_experts, int qt, void* stream_ptr, const void* ids_key) {
    if (!source || !d_x || !d_ids || !d_dst || !g_rt.copy) {
        sb_set_error("invalid Sabah MUL_MAT_ID arguments");
        return -1;
    }
    if (n_tokens == 0) {
        std::lock_guard<std::mutex> l(g_res.mu);
        ++g_res.empty_calls;
        return 0;
    }
    if (k <= 0 || rows <= 0 || n_ids <= 0 || n_tokens < 0 || n_experts <= 0 || (k % 32) != 0) {
        sb_set_error("invalid Sabah MUL_MAT_ID geometry");
        return -1;
    }
    if (x_rows <= 0 || (x_rows != 1 && x_rows != n_ids)) {
        sb_set_error("Sabah MUL_MAT_ID input rows %d must be 1 (broadcast) or n_ids %d", x_rows, n_ids);
        return -1;
    }
    if (!sb_qt_supported(qt) || k % sb_block_elems(qt) || row_stride < sb_row_bytes_of(qt, k)) {
        sb_set_error("unsupported Sabah MUL_MAT_ID quantized row (type %d, k %d, row stride %zu)", qt, k, row_stride);
        return -1;
    }
    if (!device_errors_clear()) return -1;
    cudaStream_t st = stream_ptr ? (cudaStream_t)stream_ptr : g_rt.compute;

    sb_mmid_args a{};
    a.row_stride = row_stride;
    a.x = (const float*)d_x;
    a.x_id_stride = x_id_stride;
    a.x_rows = x_rows;
    a.x_token_stride = x_token_stride;
    a.n_ids = n_ids;
    a.n_tokens = n_tokens;
    a.dst = d_dst;
    a.dst_id_stride = dst_id_stride;
    a.dst_token_stride = dst_token_stride;
    a.rows = rows;
    a.k = k;
    a.qt = qt;
    a.err = g_rt.err_d;

    uint64_t call_no;
    {
        std::lock_guard<std::mutex> l(g_res.mu);
        ++g_res.epoch;
        call_no = ++g_res.calls;
        g_res.tokens += (uint64_t)n_tokens;
    }

    // ---- extension: resident bank in device memory, ids stay on the device
    if (is_device_pointer(source)) {
        a.ex.base = (const uint8_t*)source;
        a.ex.expert_stride = expert_stride;
        a.ex.ids = (const int32_t*)d_ids;
        a.ex.ids_id_stride = ids_id_stride;
        a.ex.ids_token_stride = ids_token_stride;
        a.ex.n_experts = n_experts;
        if (sb_launch_mmid(a, st) != 0) return -1;
        std::lock_guard<std::mutex> l(g_res.mu);
        ++g_res.device_calls;
        if (g_res.sc_k > 0) {
            const size_t ids_bytes = (size_t)(n_ids - 1) * ids_id_stride + (size_t)(n_tokens - 1) * ids_token_stride + 4;
            std::vector<uint8_t> ids(ids_bytes);
            cudaStreamSynchronize(st);
            cudaMemcpy(ids.data(), d_ids, ids_bytes, cudaMemcpyDeviceToHost);
            selfcheck(source, true, a, (const int32_t*)ids.data(), ids_id_stride, ids_token_stride, expert_stride, st,
                      call_no);
        }
        status_write();
        return 0;
    }

    // ---- host-backed source (the llama.cpp contract): routing must be known on
    // the host to make the experts resident, so the ids are downloaded here
    const size_t ids_bytes = (size_t)(n_ids - 1) * ids_id_stride + (size_t)(n_tokens - 1) * ids_token_stride + 4;
    static const void* last_key = nullptr;
    static size_t last_bytes = 0;
    static uint64_t group_len = 0;
    const bool reuse = ids_key != nullptr && ids_key == last_key && ids_bytes == last_bytes && group_len < kIdGroupMax;
    group_len = reuse ? group_len + 1 : 1;
    if (!reuse) {
        if (!ids_buffer(ids_bytes)) return -1;
        SB_CUDA(cudaMemcpyAsync(g_scr.ids_h, d_ids, ids_bytes, cudaMemcpyDeviceToHost, st), "router id download");
        SB_CUDA(cudaStreamSynchronize(st), "router id synchronize");
    }
    last_key = ids_key;
    last_bytes = ids_bytes;
    const uint8_t* ids_raw = (const uint8_t*)g_scr.ids_h;

    const size_t n_slots = (size_t)n_ids * n_tokens;
    std::vector<const void*> ptrs(n_slots);
    std::vector<Fetch> miss;
    std::set<uint64_t> wait_epochs;
    const uint64_t shape = ((uint64_t)(uint32_t)qt << 56) ^ ((uint64_t)(uint32_t)rows << 32) ^
                           ((uint64_t)(uint32_t)k << 8) ^ (uint64_t)row_stride * 0x9E3779B97F4A7C15ull;
    {
        std::lock_guard<std::mutex> l(g_res.mu);
        if (reuse) {
            ++g_res.id_reuse;
            g_res.id_group_max = std::max(g_res.id_group_max, group_len);
        }
        if (g_res.capacity == 0) g_res.capacity = hot_bytes_config();
        for (int t = 0; t < n_tokens; ++t) {
            for (int i = 0; i < n_ids; ++i) {
                int e = *(const int32_t*)(ids_raw + (size_t)t * ids_token_stride + (size_t)i * ids_id_stride);
                if (e < 0 || e >= n_experts) {
                    sb_set_error("Sabah expert id out of range");
                    return -1;
                }
#if SABAH_SENTINEL == 1
                if (i == 0) e = (e + 1) % n_experts;   // test-only build: neighbouring expert
#endif
                void* d = slot_locked(source, e, (const uint8_t*)source + (size_t)e * expert_stride, expert_stride,
                                      shape, miss, wait_epochs);
                if (!d) return -1;
                ptrs[(size_t)t * n_ids + i] = d;
            }
        }
        // learn the call chain: close the previous call's edge, then, when
        // merging, reserve the followers' experts in this call's wave
        std::vector<int32_t> ids_now((size_t)n_slots);
        for (int t = 0; t < n_tokens; ++t)
            for (int i = 0; i < n_ids; ++i)
                ids_now[(size_t)t * n_ids + i] =
                    *(const int32_t*)(ids_raw + (size_t)t * ids_token_stride + (size_t)i * ids_id_stride);
        if (g_chain.prev && g_chain.prev != source) {
            ChainLink& l = g_chain.links[g_chain.prev];
            l.next = source;
            l.stride = expert_stride;
            l.shape = shape;
            l.n_experts = n_experts;
            l.shares_ids = g_chain.prev_ids == ids_now;
        }
        if (layer_merge_enabled()) {
            const void* f = source;
            for (int depth = 0; depth < 2; ++depth) {   // the layer's up to two followers
                auto li = g_chain.links.find(f);
                if (li == g_chain.links.end() || !li->second.shares_ids || !li->second.next) break;
                const ChainLink l = li->second;
                for (int32_t e : ids_now) {
                    if (e < 0 || e >= l.n_experts) continue;
                    const size_t before = miss.size();
                    if (!slot_locked(l.next, e, (const uint8_t*)l.next + (size_t)e * l.stride, l.stride, l.shape, miss,
                                     wait_epochs))
                        return -1;
                    g_chain.merged_slots += miss.size() - before;
                }
                f = l.next;
            }
        } else if (sb_pf_enabled() && n_tokens <= kPfMaxTokens) {
            // staging readahead (ref sabah_rt.cu:1517-1860): the followers' experts
            // that the tier does not hold are read into pinned buffers now, while
            // this call's fill and kernel run; their calls take the bytes from there
            const void* f = source;
            for (int depth = 0; depth < 2; ++depth) {
                auto li = g_chain.links.find(f);
                if (li == g_chain.links.end() || !li->second.shares_ids || !li->second.next) break;
                const ChainLink l = li->second;
                std::set<int32_t> distinct(ids_now.begin(), ids_now.end());
                for (int32_t e : distinct) {
                    if (e < 0 || e >= l.n_experts) continue;
                    if (g_res.map.count(Key{l.next, e, l.stride, l.shape})) continue;   // resident already
                    sb_pf_offer((const uint8_t*)l.next + (size_t)e * l.stride, l.stride);
                }
                f = l.next;
            }
        }
        g_chain.prev = source;
        g_chain.prev_ids.swap(ids_now);
        if (!fill_locked(miss, wait_epochs)) return -1;
    }
    void** d_ptrs = nullptr;
    if (!ptr_table(n_slots * sizeof(void*), &d_ptrs)) return -1;
    // one reusable table: the upload is ordered on the compute stream after the
    // previous call's kernel, which may still read it
    SB_CUDA(cudaMemcpyAsync(d_ptrs, ptrs.data(), n_slots * sizeof(void*), cudaMemcpyHostToDevice, st),
            "pointer table upload");
    if (!g_scr.ready) SB_CUDA(cudaEventCreateWithFlags(&g_scr.ready, cudaEventDisableTiming), "copy event");
    SB_CUDA(cudaEventRecord(g_scr.ready, g_rt.copy), "copy event record");
    SB_CUDA(cudaStreamWaitEvent(st, g_scr.ready, 0), "compute wait");

    a.ex.ptrs = (const void* const*)d_ptrs;
    if (sb_launch_mmid(a, st) != 0) return -1;
    {
        std::lock_guard<std::mutex> l(g_res.mu);
        if (!record_done_locked(st)) return -1;
        selfcheck(source, false, a, (const int32_t*)ids_raw, ids_id_stride, ids_token_stride, expert_stride, st,
                  call_no);
    }
    status_write();
    return 0;
}

SABAH_API int sabah_rt_snapshot(char* buf, size_t n) { return snapshot_json(buf, n); }

SABAH_API const char* sabah_rt_build_info(void) {
    static char info[128];
    std::snprintf(info, sizeof(info), "sabah_rt abi=v2 sentinel=%d", SABAH_SENTINEL);
    return info;
}

SABAH_API int sabah_rt_host_dequant(const void* src, float* dst, int qt, int n) {
    if (!src || !dst || n < 0) return -1;
    return host_dequant((const uint8_t*)src, dst, qt, n) ? 0 : -1;
}

SABAH_API int sabah_rt_get_diag(unsigned long long* calls, unsigned long long* tokens, unsigned long long* overflow,
                                unsigned long long* verify_ok, unsigned long long* verify_fail) {
    std::lock_guard<std::mutex> l(g_res.mu);
    if (calls) *calls = g_res.calls;
    if (tokens) *tokens = g_res.tokens;
    if (overflow) *overflow = g_res.overflow;
    if (verify_ok) *verify_ok = g_res.verify_ok;
    if (verify_fail) *verify_fail = g_res.verify_fail;
    return 0;
}

SABAH_API int sabah_rt_get_metrics(unsigned long long* hits, unsigned long long* misses,
                                   unsigned long long* evictions, unsigned long long* bytes_fetched,
                                   unsigned long long* resident_bytes) {
    std::lock_guard<std::mutex> l(g_res.mu);
    if (hits) *hits = g_res.hits;
    if (misses) *misses = g_res.misses;
    if (evictions) *evictions = g_res.evictions;
    if (bytes_fetched) *bytes_fetched = g_res.bytes_fetched;
    if (resident_bytes) *resident_bytes = g_res.bytes;
    return 0;
}

// Device dequantizer through the kernels' own decoders (test entry; ref
// sabah_rt.cu:3879-3885). Synchronous on the compute stream.
SABAH_API int sabah_dequant(const void* d_src, float* d_dst, int qt, int n_rows, int row_elems) {
    if (!ensure_init()) return -1;
    if (n_rows < 0 || row_elems <= 0 || !sb_row_bytes_of(qt, row_elems)) {
        sb_set_error("unsupported dequant geometry (type %d, row %d)", qt, row_elems);
        return -1;
    }
    if (n_rows == 0) return 0;
    if (sb_launch_dequant(d_src, d_dst, qt, n_rows, row_elems, g_rt.compute) != 0) return -1;
    return sb_cuda_ok(cudaStreamSynchronize(g_rt.compute), "dequant sync") ? 0 : -1;
}

SABAH_API size_t sabah_row_bytes(int qt, int n) { return sb_row_bytes_of(qt, n); }

SABAH_API int sabah_slab_init(size_t capacity_bytes) {
    std::lock_guard<std::mutex> l(g_slab.mu);
    return g_slab.init_locked(capacity_bytes) ? 0 : -1;
}
SABAH_API void* sabah_slab_alloc(size_t bytes) {
    std::lock_guard<std::mutex> l(g_slab.mu);
    if (!g_slab.base && !g_slab.init_locked(hot_bytes_config())) return nullptr;
    return g_slab.alloc_locked(bytes);
}
SABAH_API void sabah_slab_free(void* ptr) {
    if (!ptr) return;
    std::lock_guard<std::mutex> l(g_slab.mu);
    g_slab.free_locked(ptr);
}
// Releases the pool. Resident experts that lived in it are dropped from the
// residency table first, so no entry is left pointing into freed memory.
SABAH_API void sabah_slab_destroy(void) {
    std::lock_guard<std::mutex> lr(g_res.mu);
    for (auto it = g_res.map.begin(); it != g_res.map.end();) {
        if (it->second.slab) {
            g_res.bytes -= it->second.bytes;
            g_res.lru.erase(it->second.lru);
            it = g_res.map.erase(it);
        } else {
            ++it;
        }
    }
    if (g_rt.compute) cudaStreamSynchronize(g_rt.compute);
    std::lock_guard<std::mutex> l(g_slab.mu);
    g_slab.destroy_locked();
}

// Linux counterpart of the reference's direct-I/O resolution probe: which file
// and offset a host pointer maps. Registers the file for sabah_rt_read_probe.
SABAH_API int sabah_rt_resolve_probe(void* ptr, char* buf, size_t n) {
    if (!buf || n == 0) return -1;
    buf[0] = 0;
    std::string path, why;
    uint64_t off = 0;
    if (!resolve_ptr(ptr, path, off, why)) {
        std::snprintf(buf, n, "resolved=0 reason=%s", why.c_str());
        return -1;
    }
    std::lock_guard<std::mutex> l(g_disk_mu);
    size_t idx = g_disk.size();
    for (size_t i = 0; i < g_disk.size(); ++i)
        if (g_disk[i].path == path) idx = i;
    if (idx == g_disk.size()) {
        DiskFile f;
        f.path = path;
        struct stat stt;
        if (::stat(path.c_str(), &stt) == 0) f.size = (uint64_t)stt.st_size;
        g_disk.push_back(f);
    }
    std::snprintf(buf, n, "resolved=1 file=%s offset=%llu file_size=%llu align=4096 direct_io=1 depth=8", path.c_str(),
                  (unsigned long long)off, (unsigned long long)g_disk[idx].size);
    return 0;
}

// Reads `bytes` at `off` of the first registered file with O_DIRECT and reports
// the first 8 bytes, so the direct path can be checked against the mapping.
SABAH_API int sabah_rt_read_probe(uint64_t off, size_t bytes, char* buf, size_t n) {
    if (!buf || n == 0) return -1;
    buf[0] = 0;
    std::lock_guard<std::mutex> l(g_disk_mu);
    if (g_disk.empty()) {
        std::snprintf(buf, n, "no file registered");
        return -1;
    }
    const uint64_t base = off & ~(uint64_t)4095;
    const size_t delta = (size_t)(off - base);
    const size_t len = ((delta + bytes + 4095) / 4096) * 4096;
    void* mem = nullptr;
    if (posix_memalign(&mem, 4096, len) != 0) {
        std::snprintf(buf, n, "staging allocation failed");
        return -1;
    }
    int fd = ::open(g_disk[0].path.c_str(), O_RDONLY | O_DIRECT);
    if (fd < 0) fd = ::open(g_disk[0].path.c_str(), O_RDONLY);
    ssize_t got = fd >= 0 ? ::pread(fd, mem, len, (off_t)base) : -1;
    if (fd >= 0) ::close(fd);
    if (got < (ssize_t)(delta + std::min<size_t>(bytes, 8))) {
        std::snprintf(buf, n, "read failed (got %lld of %llu)", (long long)got, (unsigned long long)(delta + bytes));
        std::free(mem);
        return -1;
    }
    const uint8_t* q = (const uint8_t*)mem + delta;
    char hex[64] = {0};
    for (int i = 0; i < 8 && (size_t)i < bytes; ++i) std::snprintf(hex + 3 * i, 4, "%02x ", q[i]);
    std::snprintf(buf, n, "read_ok bytes=%lld first8=%s", (long long)got, hex);
    std::free(mem);
    return 0;
}

// ---------------------------------------------------------------------------
// per-kernel timing (the reference's SABAH_LLAMA_EVENTS probe,
// sabah_rt.cu:3771-3825): every launch bracketed by an event pair on its own
// stream, resolved when the totals are read
// ---------------------------------------------------------------------------
namespace {
struct TimedLaunch {
    const char* name;
    cudaEvent_t a, b;
};
std::mutex g_tm_mu;
bool g_tm_on = std::getenv("SABAH_LLAMA_EVENTS") && *std::getenv("SABAH_LLAMA_EVENTS") != '0';
std::vector<TimedLaunch> g_tm_pending;
std::vector<cudaEvent_t> g_tm_free;
std::map<std::string, std::pair<unsigned long long, double>> g_tm_total;   // name -> (launches, ms)

cudaEvent_t tm_event() {
    if (!g_tm_free.empty()) {
        cudaEvent_t e = g_tm_free.back();
        g_tm_free.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

void tm_resolve_locked() {
    for (auto& t : g_tm_pending) {
        float ms = 0.f;
        cudaEventSynchronize(t.b);
        if (cudaEventElapsedTime(&ms, t.a, t.b) == cudaSuccess) {
            auto& acc = g_tm_total[t.name];
            acc.first += 1;
            acc.second += ms;
        }
        g_tm_free.push_back(t.a);
        g_tm_free.push_back(t.b);
    }
    g_tm_pending.clear();
}
}  // namespace

int sb_timing_begin(const char* name, cudaStream_t st) {
    if (!g_tm_on) return -1;
    std::lock_guard<std::mutex> l(g_tm_mu);
    TimedLaunch t{name, tm_event(), tm_event()};
    cudaEventRecord(t.a, st);
    g_tm_pending.push_back(t);
    return (int)g_tm_pending.size() - 1;
}

void sb_timing_end(int slot, cudaStream_t st) {
    if (slot < 0) return;
    std::lock_guard<std::mutex> l(g_tm_mu);
    if (slot < (int)g_tm_pending.size()) cudaEventRecord(g_tm_pending[slot].b, st);
}

// Switch per-kernel timing on (1) or off (0); switching clears the totals.
SABAH_API int sabah_rt_kernel_timing(int on) {
    std::lock_guard<std::mutex> l(g_tm_mu);
    tm_resolve_locked();
    g_tm_total.clear();
    g_tm_on = on != 0;
    return 0;
}

// Totals since timing was switched on, as JSON {"kernel": [launches, ms], ...}.
// Waits for the timed launches to finish.
SABAH_API int sabah_rt_kernel_times(char* buf, size_t n) {
    std::lock_guard<std::mutex> l(g_tm_mu);
    tm_resolve_locked();
    std::string s = "{";
    for (auto& kv : g_tm_total) {
        char item[160];
        std::snprintf(item, sizeof(item), "%s\"%s\":[%llu,%.6f]", s.size() > 1 ? "," : "", kv.first.c_str(),
                      kv.second.first, kv.second.second);
        s += item;
    }
    s += "}";
    return std::snprintf(buf, n, "%s", s.c_str());
}

// ---------------------------------------------------------------------------
// multi-layer decode: n_layers routed blocks back to back on one stream,
// x_{L+1} = x_L + y_L (residual) with x updated in place. The bank pointer
// arrays are host arrays of device pointers, one per layer; ids/w are
// [n_layers][n_tokens][n_used] on the device; h is [n_tokens][n_used][ff].
// ---------------------------------------------------------------------------
SABAH_API int sabah_moe_decode(int n_layers, const void* const* gate_banks, const void* const* up_banks,
                               const void* const* down_banks, size_t gu_expert_stride, size_t down_expert_stride,
                               int n_experts, const int32_t* d_ids, const float* d_w, float* d_x, float* d_h,
                               int d_model, int ff, int n_used, int n_tokens, int qt_gate, int qt_up, int qt_down,
                               void* stream) {
    if (!gate_banks || !up_banks || !down_banks || n_layers < 0) {
        sb_set_error("invalid moe_decode arguments");
        return -1;
    }
    if (!ensure_init()) return -1;
    if (!device_errors_clear()) return -1;
    if (n_layers > 0 && n_tokens > 0 && d_ids && d_w && d_x && d_h && n_used > 0 && n_experts > 0) {
        // every layer in one persistent launch when the shapes allow it
        sb_decode_args a{};
        a.n_layers = n_layers;
        a.gate_banks = gate_banks;
        a.up_banks = up_banks;
        a.down_banks = down_banks;
        a.gu_expert_stride = gu_expert_stride;
        a.down_expert_stride = down_expert_stride;
        a.n_experts = n_experts;
        a.ids = d_ids;
        a.w = d_w;
        a.x = d_x;
        a.h = d_h;
        a.out = d_x;
        a.accumulate = 1;
        a.d_model = d_model;
        a.ff = ff;
        a.n_used = n_used;
        a.n_tokens = n_tokens;
        a.qt_gate = qt_gate;
        a.qt_up = qt_up;
        a.qt_down = qt_down;
        a.err = g_rt.err_d;
        const int taken = sb_try_decode_iq3s(a, stream ? (cudaStream_t)stream : g_rt.compute);
        if (taken != 0) return taken > 0 ? 0 : -1;
    }
    const size_t per_layer = (size_t)n_tokens * n_used;
    for (int L = 0; L < n_layers; ++L) {
        if (sabah_moe_block_ids(gate_banks[L], up_banks[L], down_banks[L], gu_expert_stride, down_expert_stride,
                                n_experts, d_ids + L * per_layer, d_w + L * per_layer, d_x, d_x, d_h, d_model, ff,
                                n_used, n_tokens, qt_gate, qt_up, qt_down, 1, stream) != 0)
            return -1;
    }
    return 0;
}
