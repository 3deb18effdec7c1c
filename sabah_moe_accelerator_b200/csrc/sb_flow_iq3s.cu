// Barrier-free persistent IQ3_S decode for one token: every layer of a decode
// step (sabah_moe_decode), or one block (sabah_moe_block_ids with one token),
// in ONE cooperative launch, one CTA per SM.
//
// The per-layer dependency chain x_L -> h_L -> x_{L+1} is all-to-all: every
// gate/up row needs all of x_L, every down row all of h_L. The kernel of
// sb_decode_iq3s.cu meets it with a grid barrier per phase and a rebuild of
// the phase's input in every CTA afterwards (two L2 round trips per phase).
// Here the data carries its own readiness instead:
//
// * x and h live in global memory as 64-bit (value, tag) pairs, written with
//   one relaxed store each. A pair is single-copy atomic, so a reader that sees
//   the tag of layer L also sees that layer's value: one round trip, no flag,
//   no barrier. Tags are (epoch << 6) + L + 1; the epoch word is bumped by the
//   last CTA to exit, so a CUDA-graph replay never mistakes an earlier
//   launch's pairs for its own. x and h are double-buffered by layer parity.
// * A gate/up item is 8 gate rows and the same 8 up rows of one slot (a
//   stacked 16-row MMA tile) over the full row. Consumer warp w decodes group
//   w (128 weights) of every item of its CTA, two items at a time (two MMA
//   chains sharing the B fragments), so each warp does the CTA's item count of
//   groups. Items are handed out in rounds (round k: the k-th item of every
//   CTA) and numbered in slot order, so early slots finish in the first rounds
//   everywhere. The epilogue warp sums an item's 16 warp partials in fixed
//   order and publishes h = silu(g) * u.
// * A down unit is 16 output rows over all n_used slots, one per CTA (d_model
//   / 16 = 128 units). Its tasks (slot, super-block) go round-robin over the
//   warps, in slot order. A task needs only its own 256 values of h: the warp
//   polls those pairs (requested during its previous task), stages them as B
//   fragments and decodes one super-block. After the layer's down stages the
//   epilogue sums the unit's task partials (super-blocks in order, then slots
//   in order, weighted) and publishes x_{L+1} = x_L + y.
// * The CTAs without a unit take more gate/up items, so that a unit CTA's
//   gate/up plus down work matches the others' gate/up work.
// * In gate/up, warp w's B fragments (group w of x) are built once per layer
//   and kept in registers for all its items.
// * Weights are inputs, so the producer warp streams tiles of the next items
//   (next layers included) while consumers wait for data.
//
// The decode core (grid lookup into fp16 subnormals with their signs +
// mma.sync with x in fp16 hi/lo parts, scale per sub-block) is sb_flow_core.cuh,
// a variant of sb_iq3s_core.cuh's with an 8-byte table of fp16 pairs.
//
// Every wait is bounded (stage barriers, sequence stamps, pair polls). A CTA
// that gives up records SB_DERR_TIMEOUT, raises a global abort word that the
// other CTAs' polls read, skips its remaining work and drains its copies.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>

#include "sb_flow_core.cuh"

namespace {

using namespace sb_iq3s;
using namespace sb_flow;

constexpr int kNC = 16;                      // consumer warps
constexpr int kProducer = kNC;               // warp 16 streams tiles
constexpr int kEpilogue = kNC + 1;           // warp 17 reduces, publishes and releases stages
constexpr int kThreads = (kNC + 2) * 32;
constexpr int kStageBytes = 16 * 880;        // a stacked gate/up tile at d_model <= 2048
constexpr int kStages = 9;                   // = issuing producer lanes: lane l owns stage l
constexpr int kMaxLayers = 64;               // tags hold the layer in 6 bits
constexpr int kMaxUsed = 16;
constexpr int kMaxDnTasks = 128;             // down tasks (slot, super-block): n_used * ff / 256
constexpr long long kPollLimit = 1ll << 21;  // pair polls (~1 us each)
constexpr int kMaxGrid = 192;                // CTAs (one per SM)
constexpr int kMaxRounds = 64;               // gate/up items of one CTA per layer
// mbarrier waits here use a short suspend-time hint: with the 20 us hint of the
// other kernels, warps waiting on a stage whose bulk copy had landed were
// measured (globaltimer trace) to resume up to ~15 us late
constexpr int kHintNs = 200;
// Gate/up partial rows are stored row-major so that the epilogue reads a
// row's 16 warp partials with 16-byte loads; the padded stride keeps 8
// consecutive rows on 8 distinct 4-bank groups (conflict-free accesses)
constexpr int kRedStride = kNC + 4;

struct Desc {
    int seq;    // sequence number of the stage's current contents
    int bad;    // bit t: tile t of the stage has an id outside [0, n_experts)
    int a, b;   // gate/up: slot, 8-row block; down: first slot, tiles
};

// A stage's use ends in two steps: its consumers arrive on done[s] (16
// arrivals per use) once their partial rows are in shared memory; the
// epilogue warp then reduces them and arrives on empty[s] for the producer.
struct Smem {
    static constexpr int table = 0;
    static constexpr int stages = table + kGridBytes;
    static constexpr int red = stages + kStages * kStageBytes;          // [kStages][16 rows][kRedStride] float
    static constexpr int dred = red + kStages * 16 * kRedStride * 4;   // [kMaxDnTasks][16 rows] float
    static constexpr int bst = dred + kMaxDnTasks * 16 * 4;            // [kNC][2 groups][32][16 B] B staging
    static constexpr int desc = bst + kNC * 1024;                      // [kStages] Desc
    static constexpr int abort_flag = desc + kStages * (int)sizeof(Desc);
    static constexpr int bars = (abort_flag + 4 + 7) & ~7;             // full, empty, done [kStages] each
    static constexpr int total = bars + 3 * kStages * 8;
};
static_assert(Smem::total <= 227 * 1024, "shared memory budget");
static_assert(Smem::stages % 128 == 0 && kStageBytes % 128 == 0, "stage alignment");
static_assert(Smem::bst % 16 == 0 && Smem::red % 16 == 0, "16-byte rows");

struct FlowLayer {
    const uint8_t* gate;
    const uint8_t* up;
    const uint8_t* down;
    const int32_t* ids;   // [n_used]
    const float* w;       // [n_used]
};

struct FlowParams {
    int n_layers, n_used, n_experts, d_model, ff;
    int rb_gu, rb_dn;          // row bytes
    int G, Gd;                 // 128-weight groups per gate/up row and per down row
    int n_gu_items;            // n_used * ff / 8
    int n_units;               // d_model / 16: CTAs [0, n_units) each own a down unit
    // Gate/up items per CTA: pu (+1 for CTAs below urem) on a unit CTA, pn (+1
    // for the first prem others) elsewhere, chosen on the host so that a unit
    // CTA's gate/up plus down work matches the others' gate/up work. Items go
    // out in rounds: round k hands the k-th item of every CTA that has one, in
    // CTA order, from round_base[k] on. Items are in slot order, so early
    // slots finish in the first rounds everywhere, and their h is published
    // long before the down tasks (also in slot order) ask for it.
    int pu, urem, pn, prem;
    int round_base[kMaxRounds + 1];
    int tps;                   // down tiles per stage (1 or 2)
    int n_dn_stages;           // ceil(n_used / tps)
    size_t gu_stride, dn_stride;
    const float* x;            // the input of block 0
    float* out;                // the last block's destination: (accumulate ? out : 0) + y
    int accumulate;
    float* h;                  // [n_used][ff]: h of the last block
    unsigned long long* xpairs;   // [2][d_model]
    unsigned long long* hpairs;   // [2][n_used][ff]
    unsigned* ctl;             // [0] epoch, [1] CTAs exited, [2] global abort; [64..) never written
    int* err;
    // test only (SABAH_TEST_FLOW_STALL): CTA 0 first waits, with a short poll
    // limit, for pairs that nothing writes, so the kernel must give up, record
    // SB_DERR_TIMEOUT and return; the next call runs clean
    int stall_test;
    int l2_prefetch;   // producer lanes warm L2 with their next tiles (SABAH_IQ3S_FLOW_L2=1; measured slower, off)
    FlowLayer layer[kMaxLayers];
};

// consumers and the epilogue warp (not the producer, which leaves early)
__device__ inline void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"((kNC + 1) * 32) : "memory"); }
__device__ inline void mbar_arrive_n(uint32_t bar, uint32_t n) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(n) : "memory");
}

__device__ inline unsigned ld_relaxed_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ inline void st_relaxed_u32(unsigned* p, unsigned v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ inline void st_pair(unsigned long long* p, float v, unsigned tag) {
    const unsigned long long u = ((unsigned long long)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(u) : "memory");
}

// This CTA gives up: local and global abort flags, and the error word.
__device__ inline void give_up(volatile int* abort_flag, unsigned* gabort, int* err) {
    *abort_flag = 1;
    st_relaxed_u32(gabort, 1u);
    if (err) atomicExch(err, SB_DERR_TIMEOUT);
}
// Another CTA's give-up is adopted as this CTA's own, so its local waits
// (stage barriers, stamps) end at once too.
__device__ inline bool aborting(volatile int* abort_flag, const unsigned* gabort) {
    if (*abort_flag) return true;
    if (ld_relaxed_u32(gabort)) {
        *abort_flag = 1;
        return true;
    }
    return false;
}
// Warp-uniform forms: every lane of the warp gets the same answer, so the
// warp never splits before a shuffle, a vote or mma.sync.
__device__ inline bool warp_aborting(volatile int* abort_flag, const unsigned* gabort) {
    return __any_sync(0xffffffffu, aborting(abort_flag, gabort));
}
__device__ inline bool warp_wait_stage(const int* stamp, int seq, uint32_t full, uint32_t parity, int* err,
                                       volatile int* abort_flag) {
    const bool stamped = __all_sync(0xffffffffu, wait_seq(stamp, seq, err, abort_flag));
    return stamped && __all_sync(0xffffffffu, mbar_wait<kHintNs>(full, parity, err, abort_flag));
}

// Warp-cooperative: lane l reads pairs [4l, 4l + 4) at p and returns their
// values once all 32 lanes see `tag` on all four. False if the kernel is
// aborting or the wait gives up.
__device__ inline bool poll4(const unsigned long long* p, unsigned tag, float4& out, volatile int* abort_flag,
                             unsigned* gabort, int* err, long long limit = kPollLimit) {
    const unsigned long long* q = p + 4 * (threadIdx.x & 31);
    for (long long i = 0; i < limit; ++i) {
        unsigned long long v0, v1, v2, v3;
        asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(v0), "=l"(v1) : "l"(q) : "memory");
        asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(v2), "=l"(v3) : "l"(q + 2) : "memory");
        const bool ok = (unsigned)(v0 >> 32) == tag && (unsigned)(v1 >> 32) == tag && (unsigned)(v2 >> 32) == tag &&
                        (unsigned)(v3 >> 32) == tag;
        if (__all_sync(0xffffffffu, ok)) {
            out = make_float4(__uint_as_float((unsigned)v0), __uint_as_float((unsigned)v1),
                              __uint_as_float((unsigned)v2), __uint_as_float((unsigned)v3));
            return true;
        }
        if ((i & 7) == 7 && __any_sync(0xffffffffu, aborting(abort_flag, gabort))) return false;
        __nanosleep(64);
    }
    if ((threadIdx.x & 31) == 0) give_up(abort_flag, gabort, err);
    return false;
}

// Lane l's 8 pairs of a 256-value piece of h at q: pairs [4l, 4l + 4) of each
// 128-value half, requested now and checked later
__device__ inline void request_pairs(const unsigned long long* q, unsigned long long (&pv)[8]) {
    q += 4 * (threadIdx.x & 31);
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(pv[0]), "=l"(pv[1]) : "l"(q) : "memory");
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(pv[2]), "=l"(pv[3]) : "l"(q + 2) : "memory");
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(pv[4]), "=l"(pv[5]) : "l"(q + 128) : "memory");
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(pv[6]), "=l"(pv[7]) : "l"(q + 130) : "memory");
}

__device__ inline int gu_items_of(const FlowParams& p, int cta) {
    return cta < p.n_units ? p.pu + (cta < p.urem ? 1 : 0) : p.pn + (cta - p.n_units < p.prem ? 1 : 0);
}
// the gate/up item of CTA `cta` in round k
__device__ inline int gu_item(const FlowParams& p, int cta, int k) {
    if (cta < p.n_units) return p.round_base[k] + cta;
    const int units_in_round = k < p.pu ? p.n_units : (k == p.pu ? p.urem : 0);
    return p.round_base[k] + units_in_round + (cta - p.n_units);
}

// The tiles of this CTA's sequence number n: gate/up items (a stacked tile: 8
// gate rows, then the same 8 up rows) and down stages (16 rows of the CTA's
// unit for up to tps consecutive slots). Fills the descriptor (bad tiles get
// their bit and no source) and the copies: source, bytes, offset in the stage.
struct Tiles {
    const uint8_t* src[2];
    uint32_t bytes[2], off[2];
    int n;
};
__device__ inline Tiles stage_tiles(const FlowParams& p, int cta, int n, int per, int ng, Desc& d) {
    const int L = n / per, idx = n % per;
    const FlowLayer& lb = p.layer[L];
    Tiles t{};
    d.bad = 0;
    if (idx < ng) {
        const int item = gu_item(p, cta, idx);
        const int rpb = p.ff / 8;
        d.a = item / rpb;
        d.b = item % rpb;
        int id = lb.ids[d.a];
#if SABAH_SENTINEL == 1
        if (d.a == 0 && id >= 0 && id < p.n_experts) id = (id + 1) % p.n_experts;   // test-only build
#endif
        t.n = 2;
        if (id < 0 || id >= p.n_experts) {
            d.bad = 1;
        } else {
            const size_t o = (size_t)id * p.gu_stride + (size_t)d.b * 8 * p.rb_gu;
            t.src[0] = lb.gate + o;
            t.src[1] = lb.up + o;
            t.bytes[0] = t.bytes[1] = 8u * p.rb_gu;
            t.off[1] = 8u * p.rb_gu;
        }
    } else {
        const int ds = idx - ng;
        d.a = ds * p.tps;
        d.b = min(p.tps, p.n_used - d.a);
        t.n = d.b;
        for (int k = 0; k < t.n; ++k) {
            int id = lb.ids[d.a + k];
#if SABAH_SENTINEL == 1
            if (d.a + k == 0 && id >= 0 && id < p.n_experts) id = (id + 1) % p.n_experts;
#endif
            if (id < 0 || id >= p.n_experts) {
                d.bad |= 1 << k;
            } else {
                t.src[k] = lb.down + (size_t)id * p.dn_stride + (size_t)cta * 16 * p.rb_dn;
                t.bytes[k] = 16u * p.rb_dn;
                t.off[k] = (uint32_t)k * 16u * p.rb_dn;
            }
        }
    }
    return t;
}

__device__ inline void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1) k_flow_iq3s(const __grid_constant__ FlowParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x;
    uint64_t* bars = (uint64_t*)(smem + Smem::bars);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kStages), done0 = smem_u32(bars + 2 * kStages);
    volatile int* abort_flag = (volatile int*)(smem + Smem::abort_flag);
    Desc* descs = (Desc*)(smem + Smem::desc);
    unsigned* gabort = p.ctl + 2;

    const int ng = gu_items_of(p, cta);                        // gate/up items of this CTA per layer
    const int nd = cta < p.n_units ? p.n_dn_stages : 0;       // down stages of this CTA per layer
    const int per = ng + nd;

    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);     // the epilogue warp, once per use
            mbar_init(done0 + 8 * s, kNC);    // 16 arrivals per use (see the consumers)
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < kStages) descs[threadIdx.x].seq = -1;
    __syncthreads();

    if (warp == kProducer) {
        // ------------------------------------------------------------ producer
        // lane l issues this CTA's sequence numbers n = l, l + kStages, ...
        // over all layers, always into stage l
        if (lane < kStages) {
            const uint32_t st0 = smem_u32(smem + Smem::stages);
            const int total = p.n_layers * per;
            int last = -1;
            for (int n = lane; n < total; n += kStages) {
                if (aborting(abort_flag, gabort)) break;
                const int s = n % kStages;
                if (n >= kStages && !mbar_wait<kHintNs>(empty0 + 8 * s, ((n / kStages) - 1) & 1, p.err, abort_flag)) break;
                Desc d;
                const Tiles t = stage_tiles(p, cta, n, per, ng, d);
                d.seq = -1;
                descs[s] = d;
                __threadfence_block();
                *(volatile int*)&descs[s].seq = n;   // the stage's previous use is released
                uint32_t tot = 0;
                for (int k = 0; k < t.n; ++k) tot += t.bytes[k];
                if (tot) {
                    mbar_expect_tx(full0 + 8 * s, tot);
                    for (int k = 0; k < t.n; ++k)
                        if (t.bytes[k]) bulk_g2s(st0 + s * kStageBytes + t.off[k], t.src[k], t.bytes[k], full0 + 8 * s);
                } else {
                    mbar_arrive(full0 + 8 * s);
                }
                last = n;
                // while this lane waits for its stage to come free again, its next
                // tiles are already on their way into L2: the copy then hits L2
                if (p.l2_prefetch && n + kStages < total) {
                    Desc dn;
                    const Tiles tn = stage_tiles(p, cta, n + kStages, per, ng, dn);
                    for (int k = 0; k < tn.n; ++k)
                        if (tn.bytes[k]) prefetch_l2(tn.src[k], tn.bytes[k]);
                }
            }
            // never leave with a copy in flight: the last use of this lane's stage must have landed
            if (last >= 0)
                for (long long i = 0; i < kSpinLimit * (kSuspendNs / kHintNs) &&
                                    !mbar_try_wait<kHintNs>(full0 + 8 * (last % kStages),
                                                                       (last / kStages) & 1); ++i) {
                }
        }
        return;
    }

    float* red = (float*)(smem + Smem::red);
    float* dred = (float*)(smem + Smem::dred);
    const unsigned epoch = ld_relaxed_u32(p.ctl);
    const int n_tasks = p.n_used * p.Gd / 2;   // down tasks per unit: (slot, super-block)
    const float nan = __int_as_float(0x7fc00000);

    if (warp == kEpilogue) {
        // ------------------------------------------------------------ epilogue
        // walks this CTA's stage uses in order: once the 16 arrivals of a use are
        // in, gate/up: sums the warps' partial rows in warp order and publishes
        // h = silu(g) * u; every use: releases the stage to the producer. After
        // the down stages of a layer: the unit's combine, x_{L+1} = x_L + y.
        consumers_sync();
        // lane (hf, r): row r; half hf of the row's gate/up partials
        const int r = lane & 15, hf = lane >> 4;
        const int row = cta * 16 + r;
        const int spr = p.Gd / 2;   // super-blocks per down row
        float xr = 0.f;
        if (nd > 0) xr = p.accumulate ? p.out[row] : 0.f;
        bool ok = true;
        for (int L = 0; L < p.n_layers && ok; ++L) {
            const unsigned tag = (epoch << 6) + (unsigned)L + 1u;
            const FlowLayer& lb = p.layer[L];
            const float wl = lane < p.n_used ? __ldg(lb.w + lane) : 0.f;
            for (int k = 0; k < per && ok; ++k) {
                const int n = L * per + k, s = n % kStages;
                ok = __all_sync(0xffffffffu, mbar_wait<kHintNs>(done0 + 8 * s, (n / kStages) & 1, p.err, abort_flag));
                if (!ok) break;
                const Desc d = descs[s];
                if (k < ng) {
                    // row r's 16 warp partials (0 for warps past G), in a fixed order
                    const float4* q = (const float4*)(red + (s * 16 + r) * kRedStride) + 2 * hf;
                    const float4 q0 = q[0], q1 = q[1];
                    float v = ((q0.x + q0.y) + (q0.z + q0.w)) + ((q1.x + q1.y) + (q1.z + q1.w));
                    v += __shfl_xor_sync(0xffffffffu, v, 16);
                    const float u = __shfl_sync(0xffffffffu, v, (lane + 8) & 31);
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(empty0 + 8 * s);   // the tile and its partial rows are consumed
                        if (d.bad && p.err) atomicExch(p.err, SB_DERR_BAD_ID);
                    }
                    if (lane < 8) {
                        const float hv = d.bad ? nan : v / (1.f + expf(-v)) * u;
                        const size_t hrow = (size_t)d.a * p.ff + (size_t)d.b * 8 + lane;
                        st_pair(p.hpairs + (size_t)(L & 1) * p.n_used * p.ff + hrow, hv, tag);
                        p.h[hrow] = hv;
                    }
                } else {
                    if (lane == 0) {
                        mbar_arrive(empty0 + 8 * s);
                        if (d.bad && p.err) atomicExch(p.err, SB_DERR_BAD_ID);
                    }
                }
            }
            if (!ok || nd == 0) continue;
            // every task of the unit is done: super-blocks in order, slots in order
            // (weighted). The combine lies on the layer's critical path (the next
            // layer's gate/up waits for x), so half hf of the warp sums half of
            // the slots and the halves are added, first half first
            const int half = (p.n_used + 1) / 2;
            const int e_lo = hf ? half : 0, e_hi = hf ? p.n_used : half;
            float part = 0.f;
            for (int e2 = 0; e2 < (p.n_used + 1) / 2; ++e2) {
                const int e = e_lo + e2;
                const float we = __shfl_sync(0xffffffffu, wl, min(e, 31));
                if (e < e_hi) {
                    float v = 0.f;
                    for (int j2 = 0; j2 < spr; ++j2) v += dred[(e * spr + j2) * 16 + r];
                    part += we * v;
                }
            }
            const float other = __shfl_xor_sync(0xffffffffu, part, 16);
            const float tot = hf ? other + part : part + other;
            xr = xr + tot;
            __syncwarp();   // dred is read before the next layer's tasks may write it
            if (lane < 16) {
                if (L + 1 < p.n_layers)
                    st_pair(p.xpairs + (size_t)((L + 1) & 1) * p.d_model + row, xr, tag + 1u);
                else
                    p.out[row] = xr;
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        uint32_t* table = (uint32_t*)(smem + Smem::table);
        fill_grid<kNC * 32>(table);
        // the partials of warps past G are never written and sum as 0
        for (int i = threadIdx.x; i < kStages * 16 * kRedStride; i += kNC * 32) red[i] = 0.f;
        consumers_sync();
        const uint32_t tab = grid_lane(table, lane);
        const int g = lane >> 2, c = lane & 3;
        const Lane Lg = lane_init<kR>(table, p.rb_gu, lane);
        const Lane Ld = lane_init<kR>(table, p.rb_dn, lane);
        const uint32_t stages32 = smem_u32(smem + Smem::stages);
        const uint32_t bst = smem_u32(smem + Smem::bst) + 1024u * warp;
        // warp 0 supplies the arrivals of the gate/up warps that do not exist (G < 16)
        const uint32_t gu_arrivals = warp == 0 ? 1u + (uint32_t)(kNC - p.G) : 1u;

        for (int L = 0; L < p.n_layers; ++L) {
            const unsigned tag = (epoch << 6) + (unsigned)L + 1u;
            const int seq0 = L * per;
            // -------------------------------------------- gate/up: group `warp` of every item, two at a time
            if (warp < p.G && ng > 0) {
                uint32_t bf[8][2];
                float inv = 0.f;
                float4 xv;
                bool have;
                if (L == 0) {
                    xv = __ldcg((const float4*)(p.x + 128 * warp) + lane);
                    have = !warp_aborting(abort_flag, gabort);
                    if (p.stall_test && cta == 0 && have)
                        have = poll4((const unsigned long long*)(p.ctl + 64), tag, xv, abort_flag, gabort, p.err,
                                     1ll << 12);
                } else {
                    have = poll4(p.xpairs + (size_t)(L & 1) * p.d_model + 128 * warp, tag, xv, abort_flag, gabort,
                                 p.err);
                }
                if (have) build_b(xv, bst, bf, inv);
                for (int k = 0; k < ng && have; k += 2) {
                    const int n0 = seq0 + k, s0 = n0 % kStages;
                    const bool two = k + 1 < ng;
                    const int n1 = n0 + 1, s1 = n1 % kStages;
                    if (!warp_wait_stage(&descs[s0].seq, n0, full0 + 8 * s0, (n0 / kStages) & 1, p.err,
                                         abort_flag) ||
                        (two && !warp_wait_stage(&descs[s1].seq, n1, full0 + 8 * s1, (n1 / kStages) & 1, p.err,
                                                 abort_flag))) {
                        have = false;
                        break;
                    }
                    const bool bad0 = descs[s0].bad != 0, bad1 = two && descs[s1].bad != 0;
                    const uint32_t t0 = stages32 + s0 * kStageBytes, t1 = stages32 + s1 * kStageBytes;
                    float a0[2] = {0.f, 0.f}, a1[2] = {0.f, 0.f};
                    if (two && !bad0 && !bad1) {
                        do_group2_q(t0, t1, warp, Lg, tab, bf, inv, a0, a1);
                    } else {
                        if (!bad0) do_group_q(t0, warp, Lg, tab, bf, inv, a0);
                        if (two && !bad1) do_group_q(t1, warp, Lg, tab, bf, inv, a1);
                    }
                    quad_sum(a0);
                    quad_sum(a1);
                    if (c == 0) {
                        float* r0 = red + (s0 * 16 + g) * kRedStride + warp;
                        r0[0] = a0[0];
                        r0[8 * kRedStride] = a0[1];
                        if (two) {
                            float* r1 = red + (s1 * 16 + g) * kRedStride + warp;
                            r1[0] = a1[0];
                            r1[8 * kRedStride] = a1[1];
                        }
                    }
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive_n(done0 + 8 * s0, gu_arrivals);
                        if (two) mbar_arrive_n(done0 + 8 * s1, gu_arrivals);
                    }
                }
            }
            // -------------------------------------------- down: tasks (slot, super-block) of this CTA's unit
            if (nd > 0 && warp < n_tasks) {
                const int spr = p.Gd / 2;   // super-blocks per down row
                const unsigned long long* hbase = p.hpairs + (size_t)(L & 1) * p.n_used * p.ff;
                // a task's 256 values of h (two 128-value pieces) are requested
                // before anything waits on them, the next task's during this one
                unsigned long long pv[8];
                request_pairs(hbase + (size_t)(warp / spr) * p.ff + 256 * (warp % spr), pv);
                for (int t = warp; t < n_tasks; t += kNC) {
                    const int e = t / spr, sb = t % spr;
                    const int ds = e / p.tps, n = seq0 + ng + ds, s = n % kStages;
                    bool ready = true;
#pragma unroll
                    for (int k = 0; k < 8; ++k) ready = ready && (unsigned)(pv[k] >> 32) == tag;
                    float4 hv[2];
                    if (__all_sync(0xffffffffu, ready)) {
#pragma unroll
                        for (int k = 0; k < 2; ++k)
                            hv[k] = make_float4(__uint_as_float((unsigned)pv[4 * k]), __uint_as_float((unsigned)pv[4 * k + 1]),
                                                __uint_as_float((unsigned)pv[4 * k + 2]),
                                                __uint_as_float((unsigned)pv[4 * k + 3]));
                    } else if (!poll4(hbase + (size_t)e * p.ff + 256 * sb, tag, hv[0], abort_flag, gabort, p.err) ||
                               !poll4(hbase + (size_t)e * p.ff + 256 * sb + 128, tag, hv[1], abort_flag, gabort, p.err)) {
                        break;
                    }
                    const float inv0 = stage_b(hv[0], bst), inv1 = stage_b(hv[1], bst + 512u);
                    __syncwarp();
                    if (t + kNC < n_tasks)   // overlaps this task's decode
                        request_pairs(hbase + (size_t)((t + kNC) / spr) * p.ff + 256 * ((t + kNC) % spr), pv);
                    if (!warp_wait_stage(&descs[s].seq, n, full0 + 8 * s, (n / kStages) & 1, p.err, abort_flag))
                        break;
                    const Desc d = descs[s];
                    const int tl = e - d.a;
                    const bool bad = (d.bad >> tl) & 1;
                    float acc[2] = {0.f, 0.f};
                    if (!bad)
                        do_superblock(stages32 + s * kStageBytes + (uint32_t)tl * 16u * p.rb_dn + (uint32_t)sb * 110u, Ld,
                                      tab, bst, inv0, bst + 512u, inv1, acc);
                    quad_sum(acc);
                    if (c == 0) {
                        dred[t * 16 + g] = bad ? nan : acc[0];
                        dred[t * 16 + g + 8] = bad ? nan : acc[1];
                    }
                    __syncwarp();   // the staging area is read; dred is written
                    if (lane == 0) {
                        // 16 arrivals per stage use: the stage's first task brings the missing ones
                        const int first = d.a * spr, in_stage = d.b * spr;
                        mbar_arrive_n(done0 + 8 * s, t == first ? 1u + (uint32_t)(kNC - in_stage) : 1u);
                    }
                }
            }
        }
    }

    // a CTA whose own wait gave up tells the others (their polls read the word)
    if (*abort_flag && lane == 0) st_relaxed_u32(gabort, 1u);
    // the last CTA out advances the epoch and clears the exit count and the abort word
    consumers_sync();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(p.ctl + 1, 1u) == gridDim.x - 1) {
            p.ctl[1] = 0;
            p.ctl[2] = 0;
            p.ctl[0] = p.ctl[0] + 1u;
            __threadfence();
        }
    }
}

// ------------------------------------------------------------------ host side
struct FlowScratch {
    void* mem = nullptr;
    bool stale = false;
};
FlowScratch g_fs;
constexpr size_t kCtlBytes = 2048;   // words 0-2 used; bytes 256 .. 1279 read by the stall test, never written
constexpr size_t kXPairBytes = 2 * 2048 * 8;
constexpr size_t kHPairBytes = 2 * (size_t)kMaxUsed * 2048 * 8;
constexpr int kMaxDev = 64;
bool g_flow_attr[kMaxDev] = {};
int g_flow_grid[kMaxDev] = {};

bool flow_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* v = std::getenv("SABAH_IQ3S_FLOW");
        on = !(v && *v == '0');
    }
    return on != 0;
}

bool a16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

void sb_flow_scratch_invalidate() { g_fs.stale = g_fs.mem != nullptr; }

int sb_try_flow_iq3s(const sb_decode_args& a, cudaStream_t st) {
    if (!flow_enabled()) return 0;
    if (a.qt_gate != SB_IQ3_S || a.qt_up != SB_IQ3_S || a.qt_down != SB_IQ3_S) return 0;
    if (a.n_tokens != 1 || a.xrows || a.n_layers < 1 || a.n_layers > kMaxLayers) return 0;
    if (a.n_used < 1 || a.n_used > kMaxUsed) return 0;
    if (a.d_model % 512 || a.d_model > 2048 || a.ff % 256 || a.ff > 2048) return 0;
    if (a.n_layers > 1 && (a.out != a.x || !a.accumulate)) return 0;   // the residual chain
    if (!a.out || !a.h || !a16(a.x) || !a16(a.out)) return 0;
    if (a.gu_expert_stride % 16 || a.down_expert_stride % 16) return 0;
    FlowParams p{};
    p.rb_gu = (int)sb_row_bytes_of(SB_IQ3_S, a.d_model);
    p.rb_dn = (int)sb_row_bytes_of(SB_IQ3_S, a.ff);
    if (16 * p.rb_gu > kStageBytes || 16 * p.rb_dn > kStageBytes || (8 * p.rb_gu) % 16) return 0;
    p.G = a.d_model / 128;
    p.Gd = a.ff / 128;
    if (a.n_used * p.Gd / 2 > kMaxDnTasks) return 0;
    for (int L = 0; L < a.n_layers; ++L)
        for (const void* b : {a.gate_banks[L], a.up_banks[L], a.down_banks[L]})
            if (!b || !a16(b)) return 0;

    int dev = 0;
    if (!sb_cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return -1;
    if (dev < 0 || dev >= kMaxDev) return 0;
    if (!g_flow_attr[dev]) {
        if (!sb_cuda_ok(cudaFuncSetAttribute(k_flow_iq3s, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem::total),
                        "flow smem attribute"))
            return -1;
        int sms = 0, per_sm = 0;
        if (!sb_cuda_ok(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count")) return -1;
        if (!sb_cuda_ok(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_flow_iq3s, kThreads, Smem::total),
                        "flow occupancy"))
            return -1;
        g_flow_grid[dev] = sms * std::min(per_sm, 1);
        g_flow_attr[dev] = true;
    }
    const int grid = g_flow_grid[dev];
    p.n_units = a.d_model / 16;
    if (grid < p.n_units || grid > kMaxGrid) return 0;   // every down unit needs a CTA of its own
    // Gate/up items per CTA. A unit CTA also runs n_used * Gd down groups, a
    // gate/up item is G groups: the CTAs without a unit take about that many
    // more items (in groups), so the down units, and with them the next
    // layer's x rows, finish together.
    {
        const int n_items = a.n_used * a.ff / 8, units = p.n_units, rest = grid - units;
        const double extra = (double)(a.n_used * p.Gd) / p.G;   // a unit's down work, in items
        double per_unit = std::floor((n_items - rest * extra) / grid + 0.5);
        if (const char* v = std::getenv("SABAH_IQ3S_FLOW_GU_PER_UNIT"))   // tuning override
            if (*v) per_unit = std::atof(v);
        long unit_items = rest == 0 ? n_items : std::lround(per_unit * units);
        unit_items = std::max(0l, std::min(unit_items, (long)n_items));
        p.pu = (int)(unit_items / units);
        p.urem = (int)(unit_items % units);
        const int left = n_items - (int)unit_items;
        p.pn = rest > 0 ? left / rest : 0;
        p.prem = rest > 0 ? left % rest : 0;
        const int rounds = std::max(p.pu + (p.urem > 0), p.pn + (p.prem > 0));
        if (rounds > kMaxRounds) return 0;
        p.round_base[0] = 0;
        for (int k = 0; k < rounds; ++k) {
            const int n = (k < p.pu ? units : k == p.pu ? p.urem : 0) + (k < p.pn ? rest : k == p.pn ? p.prem : 0);
            p.round_base[k + 1] = p.round_base[k] + n;
        }
        if (p.round_base[rounds] != n_items) return 0;
    }

    if (!g_fs.mem) {
        if (!sb_cuda_ok(cudaMalloc(&g_fs.mem, kCtlBytes + kXPairBytes + kHPairBytes), "flow scratch")) return -1;
        if (!sb_cuda_ok(cudaMemset(g_fs.mem, 0, kCtlBytes + kXPairBytes + kHPairBytes), "flow scratch reset"))
            return -1;
    } else if (g_fs.stale) {
        // a launch that gave up may have left the exit count or the abort word
        // set; the epoch (word 0) keeps counting so old pairs never match
        if (!sb_cuda_ok(cudaMemsetAsync((uint8_t*)g_fs.mem + 4, 0, 8, st), "flow scratch reset")) return -1;
    }
    g_fs.stale = false;
    uint8_t* b = (uint8_t*)g_fs.mem;
    p.ctl = (unsigned*)b;
    p.xpairs = (unsigned long long*)(b + kCtlBytes);
    p.hpairs = (unsigned long long*)(b + kCtlBytes + kXPairBytes);

    p.n_layers = a.n_layers;
    p.n_used = a.n_used;
    p.n_experts = a.n_experts;
    p.d_model = a.d_model;
    p.ff = a.ff;
    p.n_gu_items = a.n_used * a.ff / 8;
    p.tps = (2 * 16 * p.rb_dn <= kStageBytes && p.Gd <= kNC) ? 2 : 1;   // a stage's tasks (tps * Gd / 2) <= 16
    p.n_dn_stages = (a.n_used + p.tps - 1) / p.tps;
    p.gu_stride = a.gu_expert_stride;
    p.dn_stride = a.down_expert_stride;
    p.x = a.x;
    p.out = a.out;
    p.accumulate = a.accumulate;
    p.h = a.h;
    p.err = a.err;
    {
        const char* t = std::getenv("SABAH_TEST_FLOW_STALL");
        p.stall_test = t && *t == '1';
        const char* l2 = std::getenv("SABAH_IQ3S_FLOW_L2");
        p.l2_prefetch = l2 && *l2 == '1';
    }
    for (int L = 0; L < a.n_layers; ++L) {
        p.layer[L].gate = (const uint8_t*)a.gate_banks[L];
        p.layer[L].up = (const uint8_t*)a.up_banks[L];
        p.layer[L].down = (const uint8_t*)a.down_banks[L];
        p.layer[L].ids = a.ids + (size_t)L * a.n_used;
        p.layer[L].w = a.w + (size_t)L * a.n_used;
    }

    const int tslot = sb_timing_begin("decode_iq3s_flow", st);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Smem::total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_flow_iq3s, p);
    sb_timing_end(tslot, st);
    return sb_cuda_ok(e, "flow launch") ? 1 : -1;
}
