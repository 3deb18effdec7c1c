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
};

// Queue the host-to-device copies of n fills on `copy` (pinned sources
// directly, others through the staging ring). Returns once every copy is
// queued; false with the error set on failure.
bool sb_stage_fill(const sb_fill* f, int n, cudaStream_t copy);
void sb_stage_stats_get(sb_stage_stats* s);
// Stop the reader lanes and release the ring (sabah_rt_shutdown).
void sb_stage_shutdown();
