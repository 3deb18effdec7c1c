// Hot-tier fill through pinned staging (sb_staging.cu); used by the residency
// code of sb_runtime.cu.
#pragma once

#include "sb_common.cuh"

struct sb_fill {
    void* dst;          // device slot
    const void* src;    // host source (pinned, pageable or file-mapped)
    size_t bytes;
};

struct sb_stage_stats {
    unsigned long long staged_bytes;          // copied through the pinned staging ring
    unsigned long long pinned_bytes;          // copied straight from pinned sources
    unsigned long long direct_io_reads;       // chunks read from their file with O_DIRECT
    unsigned long long direct_io_bytes;
    unsigned long long direct_io_fallbacks;   // O_DIRECT reads that fell back to the mapping
    unsigned long long waves;                 // staged fills (one per call with pageable misses)
    // staging readahead (sb_pf_*)
    unsigned long long pf_reads, pf_read_bytes;   // experts read ahead into pinned buffers
    unsigned long long pf_used, pf_used_bytes;    // misses served from a readahead buffer
    unsigned long long pf_dropped;                // offers refused: every buffer busy
    unsigned long long pf_stale;                  // unclaimed readaheads overwritten by newer offers
    unsigned long long pf_waits, pf_wait_ns;      // misses that waited for a read in flight, and how long
    unsigned long long pf_wait_timeouts;          // waits that gave up (the miss was then staged as usual)
};

// Queue the host-to-device copies of n fills on `copy` (pinned sources
// directly, others through the staging ring). Returns once every copy is
// queued; false with the error set on failure.
bool sb_stage_fill(const sb_fill* f, int n, cudaStream_t copy);
void sb_stage_stats_get(sb_stage_stats* s);

// Staging readahead (SABAH_LLAMA_PREFETCH=1; off by default). A call that
// knows which experts the following calls of its layer will miss offers them
// here; reader threads read their bytes (O_DIRECT from a file mapping where
// possible) into pinned readahead buffers while this call's own work runs.
// Nothing is reserved in the hot tier.
bool sb_pf_enabled();
// Queue the read of the `bytes` at host address `src` (one expert of a
// following tensor). Pinned sources and duplicates are ignored.
void sb_pf_offer(const void* src, size_t bytes);
// A miss: if a readahead buffer holds the bytes at `src`, or is still reading
// them (waited for up to 50 ms), queue their copy into `dst` on `copy` and
// return true; otherwise false, and the caller stages the miss as usual.
bool sb_pf_take(const void* src, size_t bytes, void* dst, cudaStream_t copy);
// Stop the reader lanes and release the ring (sabah_rt_shutdown).
void sb_stage_shutdown();
