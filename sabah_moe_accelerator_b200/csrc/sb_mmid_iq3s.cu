// IQ3_S routed-expert matvec on sm_100a: decode on the CUDA cores, multiply-
// accumulate on the tensor cores.
//
// Decoding an IQ3_S weight costs more instructions than its 0.43 bytes take to
// stream from HBM, so the kernel is built around instructions per weight and
// latency hiding, not around FLOPs:
//
// * Work is a sequence of "items": one 16-row tile of one expert matrix (or,
//   for gate/up, the gate tile and the up tile of the same 16 rows). A
//   producer warp streams item tiles HBM -> shared memory with cp.async.bulk
//   into a ring of stages guarded by mbarriers, and publishes a descriptor
//   (expert validity, token, slot, row tile, x-set slot) next to each stage.
// * Item i is split over `wpt` consumer warps by groups of 4 sub-blocks (128
//   weights of a row); the 12 consumer warps work on 12 / wpt items at once and
//   never meet at a CTA barrier: the last warp to finish an item (a shared
//   counter) sums the warps' partial rows in fixed order and runs the epilogue,
//   so results are deterministic.
// * A thread decodes one grid entry (4 weights) of a row into two half2
//   registers: one LDS.32 from a 16-fold replicated copy of the 512-entry grid
//   (a warp's lookups hit distinct banks pairwise), then two PRMTs place the
//   grid bytes as fp16 subnormals b * 2^-24 with their sign bits. Those are the
//   A operand of mma.sync.m16n8k16 (f16 x f16 -> f32).
// * K is permuted so one MMA covers 4 sub-blocks: quad c owns sub-block c of
//   the group, and the 8 N columns of B hold x of sub-block n/2 split into
//   fp16 hi (n even) and lo (n odd) parts, zero outside that sub-block. After
//   the 8 MMAs of a group, D[row][2c] + D[row][2c+1] is the sub-block dot, so a
//   sub-block scale is applied once per 32 weights, and hi + lo keeps the
//   products fp32-grade (~1e-7 relative).
// * x is scaled per 32-element sub-block by a power of two (max -> [2^13, 2^14));
//   that scale and the 2^24 of the subnormal encoding are undone in fp32.
//
// Three kernels share the engine: MUL_MAT_ID (v2 contract), fused gate/up +
// SwiGLU, and down + top-k weighted combine (+ residual/accumulate).
// Launches use programmatic dependent launch: a kernel's prologue (barrier
// set-up, grid-table fill) overlaps the previous kernel; router ids,
// activations and outputs are touched only after griddepcontrol.wait. Every
// wait is bounded; on timeout the CTA records an error, skips its remaining
// work and drains its copies.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <utility>

#include "sb_iq3s_core.cuh"

namespace {

using namespace sb_iq3s;

constexpr int kConsumers = 12;                   // consumer warps
constexpr int kThreads = (kConsumers + 1) * 32;  // + one producer warp
// Tile ring: kRingBytes of shared memory cut into n_stages stages of one
// 16-row tile each (8 x 14,080 B for k = 2048, 24 x 5,280 B for k = 768).
// A lane issues its bulk copies one after another (~0.34 us apiece), so
// kIssuers producer lanes each own every kIssuers-th stage; n_stages is a
// multiple of kIssuers, so a stage always belongs to the same lane and its
// mbarrier phases are waited on in order.
constexpr int kRingBytes = 9 * 14336;
constexpr int kMaxStages = 24;
constexpr int kMaxTileBytes = 16 * 880;
constexpr int kSets = 4;
constexpr int kMaxWpt = 4;
constexpr int kMaxP = 4;                         // items in flight (kConsumers / wpt, wpt >= 3)
// The wpt warps of an item leave their partial rows in the item's stage slot of
// `red` and count themselves in; the last one reads them, runs the epilogue and
// only then releases the stage, so a slot is never reused while it is read.
constexpr int kRedSlots = kMaxStages;

enum Mode { MODE_MMID = 0, MODE_GATE_UP = 1, MODE_DOWN = 2 };

struct Desc {
    int seq;       // sequence number of the tile in the stage (see the consumer wait)
    int bad;       // 0 valid, else the device error code (the epilogue emits NaN)
    int slot;      // x-fragment set
    int t, e, rt;  // token, slot (expert choice), row tile
    int which;     // gate/up: 0 gate, 1 up
};

// Per weight format: IQ3_S needs the grid table; Q8_0 needs none and gives
// its room (and the rest of the budget) to the tile ring, since its tiles are
// 2.5x larger (34,816 B for k = 2048).
constexpr int kSmemBudget = 227 * 1024;
constexpr int kFixedBytes = kSets * kSetBytes + kRedSlots * kMaxWpt * 16 * 4 + kMaxStages * (int)sizeof(Desc) +
                            kRedSlots * 4 + 8 + 2 * kMaxStages * 8;
template <int QT>
struct Fmt {
    static constexpr int table_bytes = QT == SB_IQ3_S ? kTableBytes : 0;
    static constexpr int ring_bytes = QT == SB_IQ3_S ? kRingBytes : ((kSmemBudget - kFixedBytes - 8) & ~127);
};
template <int QT>
struct Smem {
    static constexpr int table = 0;
    static constexpr int stages = table + Fmt<QT>::table_bytes;
    static constexpr int sets = stages + Fmt<QT>::ring_bytes;
    static constexpr int red = sets + kSets * kSetBytes;                  // [kRedSlots][kMaxWpt][16] floats
    static constexpr int desc = red + kRedSlots * kMaxWpt * 16 * 4;      // [kMaxStages] Desc
    static constexpr int cnt = desc + kMaxStages * (int)sizeof(Desc);    // [kRedSlots] ints
    static constexpr int abort_flag = cnt + kRedSlots * 4;
    static constexpr int bars = (abort_flag + 4 + 7) & ~7;                // full[kMaxStages], empty[kMaxStages]
    static constexpr int total = bars + 2 * kMaxStages * 8;
};
static_assert(Smem<SB_IQ3_S>::total <= kSmemBudget && Smem<SB_Q8_0>::total <= kSmemBudget, "shared memory budget");
static_assert(Smem<SB_Q8_0>::stages % 128 == 0 && Smem<SB_Q8_0>::sets % 16 == 0, "Q8_0 ring alignment");

struct Params {
    int mode;
    int n_items;           // MMID / DOWN: tiles; GATE_UP: (gate, up) tile pairs
    int per_key;           // consecutive items sharing one x vector
    int wpt, gpw, P;       // warps per item, groups per warp, items in flight (12 / wpt)
    int k, rb, rtiles;     // row length, row bytes, 16-row tiles per matrix
    int n_stages;          // ring stages (multiple of issuers, <= kMaxStages)
    int issuers;           // producer lanes; lane l owns stages l, l + issuers, ...
    int stage_bytes;       // one tile in shared memory, rounded up to 128
    // a tile arrives as `copies` bulk copies of copy_bytes, from global rows
    // copy_src bytes apart to stage offsets copy_dst apart (IQ3_S: one copy of
    // 16 rows; Q8_0: 8 copies of a row pair at a bank-spreading pair stride)
    int copies, copy_bytes, copy_src, copy_dst;
    sb_mmid_args m;
    sb_block_args b;
    float* partial;        // DOWN: [T][n_used][d_model]; GATE_UP: [T][n_used][2][ff]
    int* counters;         // DOWN: [T][d_model / 16]; GATE_UP: [T][n_used][ff / 16]; self-resetting
    int* err;
    // the down launch of a block call: the call's gate/up launch releases its
    // dependents only after its own grid dependency (the ids' writer) is done,
    // so this launch may read the ids and stream its tiles before its own wait
    int ids_ready;
};

__device__ inline void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory"); }

// The 16-row tile of item `item`, its token / slot / row tile. Gate/up items
// alternate gate (even) and up (odd) tiles of the same rows.
__device__ inline const uint8_t* item_tile(const Params& p, int item, int& which, int& t, int& e, int& rt) {
    const int rtiles = p.rtiles;
    which = 0;
    if (p.mode == MODE_GATE_UP) {
        which = item & 1;
        item >>= 1;
    }
    rt = item % rtiles;
    const int si = item / rtiles;
    const uint8_t* base;
    if (p.mode == MODE_MMID) {
        t = si / p.m.n_ids;
        e = si % p.m.n_ids;
        base = expert_ptr(p.m.ex, t, e, p.m.n_ids);
        return base ? base + (size_t)rt * 16 * p.m.row_stride : nullptr;
    }
    t = si / p.b.n_used;
    e = si % p.b.n_used;
    const sb_experts& ex = p.mode == MODE_DOWN ? p.b.down : (which ? p.b.up : p.b.gate);
    base = expert_ptr(ex, t, e, p.b.n_used);
    return base ? base + (size_t)rt * 16 * p.rb : nullptr;
}

// the x vector of key (key = item / per_key)
__device__ inline const float* key_vector(const Params& p, int key) {
    if (p.mode == MODE_MMID) {
        // key = t * x_rows + x_row; items are ((t * n_ids + i) * rtiles + rt)
        int xt = key / p.m.x_rows, xr = key % p.m.x_rows;
#if SABAH_SENTINEL == 2
        if (p.m.x_rows > 1) xr = (xr + 1) % p.m.x_rows;   // test-only: wrong input row
#endif
#if SABAH_SENTINEL == 3
        xt = (xt + 1) % p.m.n_tokens;                     // test-only: wrong token
#endif
        return (const float*)((const uint8_t*)p.m.x + (size_t)xr * p.m.x_id_stride + (size_t)xt * p.m.x_token_stride);
    }
    if (p.mode == MODE_GATE_UP) return p.b.x + (size_t)key * p.b.d_model;
    return p.b.h + (size_t)key * p.b.ff;   // DOWN: key = t * n_used + e -> h[t][e]
}

// ---------------------------------------------------------------- the kernel
template <int QT>
__global__ void __launch_bounds__(kThreads, 1) k_iq3s(const Params p) {
    using Smem = ::Smem<QT>;
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* bars = (uint64_t*)(smem + Smem::bars);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kMaxStages);
    const int ns = p.n_stages;
    volatile int* abort_flag = (volatile int*)(smem + Smem::abort_flag);
    Desc* descs = (Desc*)(smem + Smem::desc);

    // let the next kernel on the stream begin its prologue as SMs free up: at
    // once when this launch's ids are known to be final, else after its grid
    // dependency (below), so that the next launch may trust the ids
    if (p.ids_ready) asm volatile("griddepcontrol.launch_dependents;");

    // this CTA's item range
    const int i0 = (int)((long long)blockIdx.x * p.n_items / gridDim.x);
    const int i1 = (int)((long long)(blockIdx.x + 1) * p.n_items / gridDim.x);

    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < ns; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, p.wpt);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < kRedSlots) ((int*)(smem + Smem::cnt))[threadIdx.x] = 0;
    if (threadIdx.x < kMaxStages) descs[threadIdx.x].seq = -1;
    __syncthreads();

    if (warp == kConsumers) {
        // ------------------------------------------------------ producer
        // The router ids are an input that the previous kernel on the stream
        // may have written (a router that triggers its dependents early), so
        // the producer reads them only after that kernel has completed. The
        // barrier set-up above and the consumers' table fill still overlap it.
        if (!p.ids_ready) {
            asm volatile("griddepcontrol.wait;" ::: "memory");
            asm volatile("griddepcontrol.launch_dependents;");
        }
        // lane l issues sequence numbers n = l, l + kIssuers, ... (stage n % ns,
        // always the same lane for a given stage); each lane looks up its own
        // tiles' expert addresses, so those loads overlap across lanes
        if (lane < p.issuers) {
            const uint32_t st0 = smem_u32(smem + Smem::stages);
            const uint32_t bytes = 16u * p.rb;
            int last = -1;
            for (int n = lane; i0 + n < i1 && !*abort_flag; n += p.issuers) {
                const int s = n % ns;
                if (n >= ns && !mbar_wait(empty0 + 8 * s, ((n / ns) - 1) & 1, p.err, abort_flag)) break;
                const int item = i0 + n;
                Desc d;
                const uint8_t* src = item_tile(p, item, d.which, d.t, d.e, d.rt);
                d.bad = !src ? SB_DERR_BAD_ID : ((uintptr_t)src & 15) ? SB_DERR_MISALIGNED : 0;
                d.slot = (item / p.per_key) % kSets;
                d.seq = -1;
                descs[s] = d;   // published by the arrive below (release)
                __threadfence_block();
                *(volatile int*)&descs[s].seq = n;   // the stage's previous tile is released
                if (!d.bad) {
                    mbar_expect_tx(full0 + 8 * s, bytes);
                    for (int j = 0; j < p.copies; ++j)
                        bulk_g2s(st0 + s * p.stage_bytes + j * p.copy_dst, src + (size_t)j * p.copy_src, p.copy_bytes,
                                 full0 + 8 * s);
                } else {
                    mbar_arrive(full0 + 8 * s);
                }
                last = n;
            }
            // never leave with copies in flight: the last use of each of this
            // lane's stages must have landed
            for (int n = std::max(lane, last - ns + p.issuers); n <= last; n += p.issuers)
                for (long long i = 0; i < kSpinLimit && !mbar_try_wait(full0 + 8 * (n % ns), (n / ns) & 1); ++i) {
                }
        }
        return;
    }

    // ---------------------------------------------------------- consumers
    uint32_t* table = (uint32_t*)(smem + Smem::table);
    if constexpr (QT == SB_IQ3_S) fill_table<kConsumers * 32>(table);
    // activations and outputs only after the previous kernel on the stream is done
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (!p.ids_ready) asm volatile("griddepcontrol.launch_dependents;");

    const int g = lane >> 2, c = lane & 3;
    const uint32_t boff = lane_boff(lane);
    Lane L{};
    LaneQ8 LQ{};
    if constexpr (QT == SB_IQ3_S)
        L = lane_init(table, p.rb, lane);
    else
        LQ = lane_init_q8(p.rb, p.copy_dst, lane);
    const uint32_t stages32 = smem_u32(smem + Smem::stages), sets32 = smem_u32(smem + Smem::sets);
    const int pos = warp / p.wpt;   // which of the P items in flight
    const int wsub = warp % p.wpt;  // which part of the row
    float* red = (float*)(smem + Smem::red);
    int* cnt = (int*)(smem + Smem::cnt);
    uint8_t* sets = smem + Smem::sets;

    // Items are walked in chunks whose x vectors map to distinct set slots
    // (keys [kc * kSets, (kc + 1) * kSets)); sets are rebuilt at chunk starts.
    int item = i0;
    while (item < i1) {
        const int key0 = item / p.per_key;
        const int kc = key0 / kSets;
        const int chunk_end = min(i1, (kc + 1) * kSets * p.per_key);
        consumers_sync();   // all warps are done with the previous chunk's sets
        {
            const int k_last = (chunk_end - 1) / p.per_key;
            for (int key = key0; key <= k_last; ++key)
                build_set<kConsumers * 32>(key_vector(p, key), p.k, sets + (key % kSets) * kSetBytes);
        }
        consumers_sync();
        for (int it = item + pos; it < chunk_end; it += p.P) {
            const int seq = it - i0;   // one stage per item, in this CTA's order
            const int s = seq % ns;
            // The producer stamps seq into the stage descriptor only after the
            // stage's previous tile (seq - ns) was released, so once the stamp is
            // seen the parity wait refers to this tile's phase. Without it, a warp
            // running ns tiles ahead of a late copy would take the old phase's
            // completion for its own.
            const bool stamped = wait_seq(&descs[s].seq, seq, p.err, abort_flag);
            const bool landed = stamped && mbar_wait(full0 + 8 * s, (seq / ns) & 1, p.err, abort_flag);
            const Desc d = descs[s];
            const int bad = !stamped ? -1 : !landed ? SB_DERR_TIMEOUT : d.bad;
            float acc[2] = {0.f, 0.f};
            if (!bad)
                for (int q = wsub * p.gpw; q < (wsub + 1) * p.gpw; q += 2) {
                    if constexpr (QT == SB_IQ3_S)
                        do_pair(stages32 + s * p.stage_bytes, q, sets32 + d.slot * kSetBytes + boff, L, acc);
                    else
                        do_pair_q8(stages32 + s * p.stage_bytes, q, sets32 + d.slot * kSetBytes + boff, LQ, acc);
                }
            // this warp's rows: reduce the 4 quads, publish, count
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 1);
                acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 2);
            }
            float* rr = red + (s * kMaxWpt + wsub) * 16;
            if (c == 0) {
                // tile rows of (g, h): IQ3_S g and g + 8, Q8_0 2g and 2g + 1
                const int r0 = QT == SB_IQ3_S ? g : 2 * g, r1 = QT == SB_IQ3_S ? g + 8 : 2 * g + 1;
                rr[r0] = acc[0];
                rr[r1] = acc[1];
            }
            __threadfence_block();
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                last = atomicAdd(cnt + s, 1) == p.wpt - 1;
                if (last) cnt[s] = 0;
                else mbar_arrive(empty0 + 8 * s);
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (!last) continue;
            // ---- epilogue (the last warp of the item), one row per lane
            __threadfence_block();
            float v = 0.f;
            if (lane < 16)
                for (int w = 0; w < p.wpt; ++w) v += red[(s * kMaxWpt + w) * 16 + lane];
            __syncwarp();
            // the partial rows are read: the stage (and its red slot) may be reused
            if (lane == 0) mbar_arrive(empty0 + 8 * s);
            if (bad < 0) continue;   // no descriptor (the CTA is aborting; the error is recorded)
            if (lane < 16) {
                if (bad) {
                    v = __int_as_float(0x7fc00000);
                    if (lane == 0 && p.err) atomicExch(p.err, bad);
                }
                const int row = d.rt * 16 + lane;
                if (p.mode == MODE_MMID) {
                    float* dst = (float*)((uint8_t*)p.m.dst + (size_t)d.t * p.m.dst_token_stride +
                                          (size_t)d.e * p.m.dst_id_stride);
                    dst[row] = v;
                } else if (p.mode == MODE_GATE_UP) {
                    // gate and up of these rows may be decoded by different CTAs: each
                    // writes its half, the second to finish forms silu(g) * u
                    const size_t te = (size_t)d.t * p.b.n_used + d.e;
                    p.partial[(te * 2 + d.which) * p.b.ff + row] = v;
                    __threadfence();
                    __syncwarp(0x0000ffffu);
                    int fin = 0;
                    if (lane == 0) {
                        int* gc = p.counters + te * p.rtiles + d.rt;
                        fin = atomicAdd(gc, 1) == 1;
                        if (fin) *gc = 0;
                    }
                    fin = __shfl_sync(0x0000ffffu, fin, 0);
                    if (fin) {
                        __threadfence();
                        const float gv = __ldcg(p.partial + (te * 2) * p.b.ff + row);
                        const float uv = __ldcg(p.partial + (te * 2 + 1) * p.b.ff + row);
                        p.b.h[te * p.b.ff + row] = gv / (1.f + expf(-gv)) * uv;
                    }
                } else {
                    // DOWN: weighted partial; the last of the n_used slots of this
                    // row tile combines them in slot order
                    p.partial[((size_t)d.t * p.b.n_used + d.e) * p.b.d_model + row] =
                        p.b.w[(size_t)d.t * p.b.n_used + d.e] * v;
                    __threadfence();
                    __syncwarp(0x0000ffffu);
                    int fin = 0;
                    if (lane == 0) {
                        int* gc = p.counters + (size_t)d.t * p.rtiles + d.rt;
                        fin = atomicAdd(gc, 1) == p.b.n_used - 1;
                        if (fin) *gc = 0;
                    }
                    fin = __shfl_sync(0x0000ffffu, fin, 0);
                    if (fin) {
                        __threadfence();
                        float tot = 0.f;
                        for (int e = 0; e < p.b.n_used; ++e)
                            tot += __ldcg(p.partial + ((size_t)d.t * p.b.n_used + e) * p.b.d_model + row);
                        float* o = p.b.out + (size_t)d.t * p.b.d_model + row;
                        *o = p.b.accumulate ? *o + tot : tot;
                    }
                }
            }
        }
        item = chunk_end;
    }
}

// ------------------------------------------------------------------ host side
// Per device: the shared-memory attribute is set and the SM count read once
// with that device current (a process may call on more than one device).
constexpr int kMaxDevices = 64;
bool g_attr_set[kMaxDevices] = {};
int g_num_sms[kMaxDevices] = {};

// split a row of k weights (G = k / 128 groups) over wpt warps, gpw groups each
bool plan_groups(int k, int& wpt, int& gpw) {
    if (k % 128 || k > 2048) return false;
    const int G = k / 128;
    // even groups per warp: the decode walks whole super-blocks (group pairs)
    for (int w : {4, 3}) {   // P = kConsumers / w <= kMaxP
        if (kConsumers % w == 0 && kConsumers / w <= kMaxP && G % w == 0 && G / w <= 8 && (G / w) % 2 == 0) {
            wpt = w;
            gpw = G / w;
            return true;
        }
    }
    return false;
}

// Tile geometry of a format: stage size and the bulk copies that fill a stage.
template <int QT>
void tile_geometry(Params& p) {
    if (QT == SB_IQ3_S) {
        p.copies = 1;
        p.copy_bytes = 16 * p.rb;
        p.copy_src = 0;
        p.copy_dst = 0;
        p.stage_bytes = (16 * p.rb + 127) & ~127;
    } else {
        // row pairs at a stride of 12 (mod 32) words, at least 4 bytes of pad:
        // a lane's last word load may run past its pair
        const int words = 2 * p.rb / 4;
        int pad = ((12 - words % 32) + 32) % 32 * 4;
        if (pad < 4) pad += 128;
        p.copies = 8;
        p.copy_bytes = 2 * p.rb;
        p.copy_src = 2 * p.rb;
        p.copy_dst = 2 * p.rb + pad;
        p.stage_bytes = (8 * p.copy_dst + 127) & ~127;
    }
}

template <int QT>
int launch(Params& p, cudaStream_t st) {
    using Smem = ::Smem<QT>;
    int dev = 0;
    if (!sb_cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return -1;
    if (dev < 0 || dev >= kMaxDevices) {
        sb_set_error("the tensor-core matvec kernels support devices 0..%d", kMaxDevices - 1);
        return -1;
    }
    static bool attr_set[kMaxDevices] = {};
    if (!attr_set[dev]) {
        if (!sb_cuda_ok(cudaFuncSetAttribute(k_iq3s<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem::total),
                        "matvec smem attribute"))
            return -1;
        if (!g_attr_set[dev]) {
            if (!sb_cuda_ok(cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev),
                            "SM count"))
                return -1;
            g_attr_set[dev] = true;
        }
        attr_set[dev] = true;
    }
    p.P = kConsumers / p.wpt;
    tile_geometry<QT>(p);
    const int fit = Fmt<QT>::ring_bytes / p.stage_bytes;
    p.issuers = std::min(kIssuers, fit);
    if (p.issuers < 1) {
        sb_set_error("tile of %d bytes does not fit the ring", p.stage_bytes);
        return -1;
    }
    p.n_stages = std::min(kMaxStages, fit / p.issuers * p.issuers);
    const int grid = std::max(1, std::min(p.n_items, g_num_sms[dev]));
    const char* names[3][2] = {{"mmid_iq3s", "mmid_q8_0"}, {"gate_up_iq3s", "gate_up_q8_0"},
                               {"down_iq3s", "down_q8_0"}};
    const int tslot = sb_timing_begin(names[p.mode][QT == SB_IQ3_S ? 0 : 1], st);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Smem::total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_iq3s<QT>, p);
    sb_timing_end(tslot, st);
    return sb_cuda_ok(e, "matvec launch") ? 1 : -1;
}

int launch(Params& p, int qt, cudaStream_t st) {
    return qt == SB_IQ3_S ? launch<SB_IQ3_S>(p, st) : launch<SB_Q8_0>(p, st);
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// Scratch of the fused block: the partial sums that CTAs hand to the last
// finisher of a row tile (gate/up halves; the n_used weighted down partials),
// and the arrival counters, which the last finisher resets to zero. Counters
// sit in their own region at the front, so every shape uses a prefix of the
// same zeroed words; partial sums follow it. The buffer grows on demand
// (cudaMalloc outside any graph capture: the first call of a shape must come
// before capturing it) and is shared by every call, so calls of the fused
// block must not overlap on the GPU.
struct BlockScratch {
    float* gu_partial = nullptr;   // [T][n_used][2][ff]
    float* dn_partial = nullptr;   // [T][n_used][d_model]
    int* gu_counters = nullptr;    // [T][n_used][ff / 16]
    int* dn_counters = nullptr;    // [T][d_model / 16]
    void* mem = nullptr;
    size_t counter_cap = 0, partial_cap = 0;
    bool stale = false;            // a kernel gave up mid-call: counters may be left non-zero
};
BlockScratch g_bs;

bool block_scratch(int T, int n_used, int d_model, int ff, cudaStream_t st) {
    auto up256 = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t gup = up256((size_t)T * n_used * 2 * ff * 4), dnp = up256((size_t)T * n_used * d_model * 4);
    const size_t guc = up256((size_t)T * n_used * (ff / 16) * 4), dnc = up256((size_t)T * (d_model / 16) * 4);
    if (guc + dnc > g_bs.counter_cap || gup + dnp > g_bs.partial_cap) {
        const size_t ccap = std::max(guc + dnc, g_bs.counter_cap), pcap = std::max(gup + dnp, g_bs.partial_cap);
        if (g_bs.mem) {
            cudaDeviceSynchronize();   // no kernel of an earlier call may still use it
            cudaFree(g_bs.mem);
        }
        g_bs = BlockScratch{};
        if (!sb_cuda_ok(cudaMalloc(&g_bs.mem, ccap + pcap), "block scratch")) return false;
        if (!sb_cuda_ok(cudaMemset(g_bs.mem, 0, ccap), "block scratch reset")) return false;
        g_bs.counter_cap = ccap;
        g_bs.partial_cap = pcap;
    }
    if (g_bs.stale) {
        // stream-ordered: runs after every earlier kernel on this stream
        if (!sb_cuda_ok(cudaMemsetAsync(g_bs.mem, 0, g_bs.counter_cap, st), "block scratch reset")) return false;
        g_bs.stale = false;
    }
    uint8_t* b = (uint8_t*)g_bs.mem;
    g_bs.gu_counters = (int*)b;
    g_bs.dn_counters = (int*)(b + guc);
    g_bs.gu_partial = (float*)(b + g_bs.counter_cap);
    g_bs.dn_partial = (float*)(b + g_bs.counter_cap + gup);
    return true;
}

// Fixed scratch of the allocation-free block (sb_block_iq3s_fixed). Counters
// occupy the first kFixedCounterBytes whatever the shape and are cleared on
// the call's stream at the start of every call. The partial sums follow.
constexpr size_t kFixedScratchBytes = (size_t)1 << 20;    // 1 MiB
constexpr size_t kFixedCounterBytes = (size_t)64 << 10;   // 16,384 counters
constexpr int kFixedMaxDevices = kMaxDevices;
struct FixedScratch {
    uint8_t* ptr = nullptr;   // device address of sb_fixed_scratch on this device
};
FixedScratch g_fixed[kFixedMaxDevices];

bool fast_path_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* v = std::getenv("SABAH_IQ3S_MMA");
        on = !(v && *v == '0');
    }
    return on != 0;
}

}  // namespace

static __device__ __align__(256) uint8_t sb_fixed_scratch[kFixedScratchBytes];

void sb_block_scratch_invalidate() { g_bs.stale = g_bs.mem != nullptr; }

namespace {
// Tiles of this size fit the format's ring (IQ3_S: the historical 16 x 880 B cap)
bool tile_fits(int qt, size_t rb) {
    return qt == SB_IQ3_S ? 16 * rb <= (size_t)kMaxTileBytes : 16 * rb <= (size_t)Fmt<SB_Q8_0>::ring_bytes / 4;
}

int block_two_launches(const sb_block_args& a, int qt, cudaStream_t st);

int try_mmid(const sb_mmid_args& a, cudaStream_t st) {
    int wpt, gpw;
    if (!plan_groups(a.k, wpt, gpw) || a.rows % 16) return 0;
    const size_t rb = sb_row_bytes_of(a.qt, a.k);
    if (a.row_stride != rb || !tile_fits(a.qt, rb)) return 0;
    if (!a.ex.ptrs && (!aligned16(a.ex.base) || a.ex.expert_stride % 16)) return 0;
    if (a.x_id_stride % 16 || a.x_token_stride % 16 || !aligned16(a.x)) return 0;
    const long long items = (long long)a.n_ids * a.n_tokens * (a.rows / 16);
    if (items > (1ll << 30)) return 0;
    Params p{};
    p.mode = MODE_MMID;
    p.rtiles = a.rows / 16;
    p.n_items = (int)items;
    p.per_key = a.x_rows == 1 ? a.n_ids * p.rtiles : p.rtiles;
    p.wpt = wpt;
    p.gpw = gpw;
    p.k = a.k;
    p.rb = (int)rb;
    p.m = a;
    p.err = a.err;
    return launch(p, a.qt, st);
}
}  // namespace

int sb_try_mmid_iq3s(const sb_mmid_args& a, cudaStream_t st) {
    if (a.qt != SB_IQ3_S || !fast_path_enabled()) return 0;
    const int grouped = sb_try_mmid_iq3s_grouped(a, st);   // prefill-sized calls
    if (grouped != 0) return grouped;
    return try_mmid(a, st);
}

int sb_try_mmid_q8_0(const sb_mmid_args& a, cudaStream_t st) {
    if (a.qt != SB_Q8_0 || !fast_path_enabled()) return 0;
    return try_mmid(a, st);
}

int sb_try_block_iq3s(const sb_block_args& a, cudaStream_t st) {
    if (a.qt_gate != SB_IQ3_S || a.qt_up != SB_IQ3_S || a.qt_down != SB_IQ3_S || !fast_path_enabled()) return 0;
    {   // many (token, slot) pairs; gathered input rows are copied into place first
        const int grouped = sb_block_iq3s_grouped(a, st);
        if (grouped != 0) return grouped;
    }
    // one persistent launch (sb_decode_iq3s.cu, one block): every combine is CTA-local,
    // so it has none of the cross-CTA hand-offs of the two launches below
    if (!a.gate.ptrs && !a.up.ptrs && !a.down.ptrs && a.gate.ids && a.gate.ids == a.up.ids &&
        a.gate.ids == a.down.ids && a.gate.ids_id_stride == 4 && a.gate.ids_token_stride == (size_t)4 * a.n_used &&
        a.gate.expert_stride == a.up.expert_stride && a.gate.n_experts == a.down.n_experts) {
        const void* gb = a.gate.base;
        const void* ub = a.up.base;
        const void* db = a.down.base;
        sb_decode_args d{};
        d.n_layers = 1;
        d.gate_banks = &gb;
        d.up_banks = &ub;
        d.down_banks = &db;
        d.gu_expert_stride = a.gate.expert_stride;
        d.down_expert_stride = a.down.expert_stride;
        d.n_experts = a.gate.n_experts;
        d.ids = a.gate.ids;
        d.w = a.w;
        d.x = const_cast<float*>(a.x);   // read only: with one block the combine goes to out
        d.h = a.h;
        d.out = a.out;
        d.accumulate = a.accumulate;
        d.xrows = a.xrows;
        d.n_xrows = a.n_xrows;
        d.d_model = a.d_model;
        d.ff = a.ff;
        d.n_used = a.n_used;
        d.n_tokens = a.n_tokens;
        d.qt_gate = a.qt_gate;
        d.qt_up = a.qt_up;
        d.qt_down = a.qt_down;
        d.err = a.err;
        const int taken = sb_try_decode_iq3s(d, st);
        if (taken != 0) return taken;
    }
    return block_two_launches(a, SB_IQ3_S, st);
}

int sb_try_block_q8_0(const sb_block_args& a, cudaStream_t st) {
    if (a.qt_gate != SB_Q8_0 || a.qt_up != SB_Q8_0 || a.qt_down != SB_Q8_0 || !fast_path_enabled()) return 0;
    return block_two_launches(a, SB_Q8_0, st);
}

namespace {
// gate/up + SwiGLU, then down + weighted combine: one launch each, over the
// shared block scratch
int block_two_launches(const sb_block_args& a, int qt, cudaStream_t st) {
    if (a.xrows) return 0;   // the launches below read rows t only
    int wpt_g, gpw_g, wpt_d, gpw_d;
    if (!plan_groups(a.d_model, wpt_g, gpw_g) || !plan_groups(a.ff, wpt_d, gpw_d)) return 0;
    if (a.ff % 16 || a.d_model % 16) return 0;
    const size_t rbg = sb_row_bytes_of(qt, a.d_model), rbd = sb_row_bytes_of(qt, a.ff);
    if (!tile_fits(qt, rbg) || !tile_fits(qt, rbd)) return 0;
    for (const sb_experts* e : {&a.gate, &a.up, &a.down})
        if (!e->ptrs && (!aligned16(e->base) || e->expert_stride % 16)) return 0;
    if (!aligned16(a.x) || !aligned16(a.h) || (a.d_model * 4) % 16 || (a.ff * 4) % 16) return 0;
    if (!block_scratch(a.n_tokens, a.n_used, a.d_model, a.ff, st)) return -1;

    Params p{};
    p.b = a;
    p.err = a.err;
    // gate + up + SwiGLU: items (t, e, row tile, gate | up)
    p.mode = MODE_GATE_UP;
    p.rtiles = a.ff / 16;
    p.n_items = a.n_tokens * a.n_used * p.rtiles * 2;
    p.per_key = a.n_used * p.rtiles * 2;   // one x per token
    p.wpt = wpt_g;
    p.gpw = gpw_g;
    p.k = a.d_model;
    p.rb = (int)rbg;
    p.partial = g_bs.gu_partial;
    p.counters = g_bs.gu_counters;
    if (launch(p, qt, st) < 0) return -1;
    // down + weighted combine: items (t, e, row tile); launched right after the
    // gate/up launch, which released its dependents only once the ids were final
    p.mode = MODE_DOWN;
    p.ids_ready = 1;
    p.rtiles = a.d_model / 16;
    p.n_items = a.n_tokens * a.n_used * p.rtiles;
    p.per_key = p.rtiles;               // one h per (token, slot)
    p.wpt = wpt_d;
    p.gpw = gpw_d;
    p.k = a.ff;
    p.rb = (int)rbd;
    p.partial = g_bs.dn_partial;
    p.counters = g_bs.dn_counters;
    return launch(p, qt, st);
}
}  // namespace

int sb_block_iq3s_fixed(const sb_block_args& a, cudaStream_t st) {
    if (a.qt_gate != SB_IQ3_S || a.qt_up != SB_IQ3_S || a.qt_down != SB_IQ3_S) {
        sb_set_error("the allocation-free block takes IQ3_S gate, up and down only (got %d/%d/%d)", a.qt_gate,
                     a.qt_up, a.qt_down);
        return -1;
    }
    int wpt_g, gpw_g, wpt_d, gpw_d;
    if (!plan_groups(a.d_model, wpt_g, gpw_g) || !plan_groups(a.ff, wpt_d, gpw_d) || a.ff % 16 || a.d_model % 16) {
        sb_set_error("the allocation-free block needs d_model and ff each in {768, 1024, 1536, 2048} (got %d, %d)",
                     a.d_model, a.ff);
        return -1;
    }
    for (const sb_experts* e : {&a.gate, &a.up, &a.down})
        if (!aligned16(e->base) || e->expert_stride % 16) {
            sb_set_error("the allocation-free block needs 16-byte aligned banks and expert strides");
            return -1;
        }
    if (!aligned16(a.x) || !aligned16(a.h)) {
        sb_set_error("the allocation-free block needs 16-byte aligned x and h");
        return -1;
    }
    auto up256 = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t slots = (size_t)a.n_tokens * a.n_used;
    const size_t guc = up256(slots * (a.ff / 16) * 4), dnc = up256((size_t)a.n_tokens * (a.d_model / 16) * 4);
    const size_t gup = up256(slots * 2 * a.ff * 4), dnp = up256(slots * a.d_model * 4);
    if (guc + dnc > kFixedCounterBytes || gup + dnp > kFixedScratchBytes - kFixedCounterBytes) {
        sb_set_error("the allocation-free block needs %zu bytes of partial sums and %zu of counters for %d tokens x %d "
                     "slots; its fixed scratch holds %zu and %zu",
                     gup + dnp, guc + dnc, a.n_tokens, a.n_used, kFixedScratchBytes - kFixedCounterBytes,
                     kFixedCounterBytes);
        return -1;
    }
    int dev = 0;
    if (!sb_cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return -1;
    if (dev < 0 || dev >= kFixedMaxDevices) {
        sb_set_error("the allocation-free block supports devices 0..%d", kFixedMaxDevices - 1);
        return -1;
    }
    FixedScratch& fs = g_fixed[dev];
    if (!fs.ptr) {
        void* ptr = nullptr;
        if (!sb_cuda_ok(cudaGetSymbolAddress(&ptr, sb_fixed_scratch), "fixed scratch address")) return -1;
        fs.ptr = (uint8_t*)ptr;
    }
    // Every call starts from zeroed counters, queued on the call's stream: a
    // call that gave up part-way (a device error) leaves no stale counts for
    // the next one. Only this shape's counter words are cleared.
    if (!sb_cuda_ok(cudaMemsetAsync(fs.ptr, 0, guc + dnc, st), "fixed scratch clear")) return -1;

    Params p{};
    p.b = a;
    p.err = a.err;
    p.mode = MODE_GATE_UP;
    p.rtiles = a.ff / 16;
    p.n_items = a.n_tokens * a.n_used * p.rtiles * 2;
    p.per_key = a.n_used * p.rtiles * 2;
    p.wpt = wpt_g;
    p.gpw = gpw_g;
    p.k = a.d_model;
    p.rb = (int)sb_row_bytes_of(SB_IQ3_S, a.d_model);
    p.partial = (float*)(fs.ptr + kFixedCounterBytes);
    p.counters = (int*)fs.ptr;
    if (launch<SB_IQ3_S>(p, st) < 0) return -1;
    p.mode = MODE_DOWN;
    p.ids_ready = 1;   // right after the gate/up launch (see block_two_launches)
    p.rtiles = a.d_model / 16;
    p.n_items = a.n_tokens * a.n_used * p.rtiles;
    p.per_key = p.rtiles;
    p.wpt = wpt_d;
    p.gpw = gpw_d;
    p.k = a.ff;
    p.rb = (int)sb_row_bytes_of(SB_IQ3_S, a.ff);
    p.partial = (float*)(fs.ptr + kFixedCounterBytes + gup);
    p.counters = (int*)(fs.ptr + guc);
    return launch<SB_IQ3_S>(p, st) < 0 ? -1 : 0;
}
