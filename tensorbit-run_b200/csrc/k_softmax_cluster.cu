// k_softmax_cluster.cu -- f32 row softmax, each row split over the CTAs of
// one thread-block cluster, the reference's in-order sum reproduced exactly.
//
// Reference arithmetic (tb_cpu_softmax_f32, src/ops/softmax.c:4-32):
//   m = max x (strict '>', from -inf);  e_i = expf(x_i - m);
//   sum = ((e_0 + e_1) + e_2) + ...  (f32, in order);  y_i = e_i * (1.0f/sum) if sum > 0.
// Here e_i = 2^fma(x_i, log2(e), -m*log2(e)) on the MUFU pipe (one expression
// everywhere, so every pass sees the same bits; see Expo for its accuracy).
// The sum is the in-order f32 sum of those e_i, bit for bit: the integer-
// grid argument of ordered_sum.cuh, applied per 256-term tile.
//
// Layout.  A row of `cols` terms is cut into 256-term tiles; a cluster of C
// CTAs (C = ceil(tiles / 64), at most 8) takes a row, CTA c owning a segment
// of T = ceil(tiles / C) consecutive tiles (at most 64 KB).  The clusters are
// persistent: cluster q takes rows q, q + Q, ...  Each CTA has three segment
// buffers, filled by bulk asynchronous copies (cp.async.bulk, one mbarrier
// each): a segment is read from HBM once, two rows ahead of its use.
//
// Roles (16 warps per CTA):
//   workers (9 warps), per row j, three phases interleaved with the next row,
//     two tiles per warp at a time:
//     A(j)  max over the segment; the segment max goes to every CTA of the
//           cluster (st.shared::cluster + a remote mbarrier arrive);
//     B(j)  with the row max: e in place, a sum estimate per tile (integer
//           redux), the segment's estimate to every CTA;
//     A(j+1)
//     C(j)  with the estimates of the segments before this one: the running-
//           sum estimate at each tile start -> the binade the exact running
//           sum is predicted to be in -> per tile the integer sum of
//           rne(e / u) on that binade's grid u, as (D0, D1) for an even / odd
//           running sum at the tile start (they differ only when a term is an
//           exact tie), into this CTA's summary slot of the row; one remote
//           arrive tells the row's scanner; the buffer is released and the
//           row three ahead is copied into it.
//     So each cluster exchange has a whole phase of work to land in.
//   scanners (3 warps; row j's scanner is warp (j / C) % 3 of CTA j % C):
//     tile 0 summed in order by one lane; then 32 tiles per step, their
//     summaries read from the owning CTAs' shared memory (ld.shared::cluster):
//     an ordered composition scan of the (D0, D1) functions gives each tile's
//     start; the first tile that is not on its predicted grid, crosses the
//     binade or is flagged is summed term by term (ordered_sum_tile, its
//     terms recomputed from x in L2; tiles predicted to cross are loaded
//     ahead).  The row's sum and max go to every CTA.
//   finalizers (4 warps): y = e * (1/sum) of the CTA's segment of each row,
//     in row order, e recomputed from x (still in L2: the copies keep it
//     there), 16 loads in flight per thread, streaming stores.
// Every wait is bounded (%globaltimer, 2 s): a timeout raises
// TB_B200_FLAG_WAIT_TIMEOUT and the CTA skips its remaining waits; every
// thread of every CTA still reaches the final cluster barrier, so no CTA
// leaves while a peer may write its shared memory, and no copy is in flight
// when a CTA exits.  Only this GPU's memory is read; no multicast.
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <stddef.h>

#include <type_traits>

#include "ordered_sum.cuh"
#include "tb_device.cuh"
#include "tb_internal.h"
#include "tma.cuh"

namespace {

constexpr int kTileN = 256;
constexpr int kSegTiles = 64;  // tiles per CTA segment, at most
constexpr int kMaxC = 8;       // CTAs per cluster (portable limit)
constexpr int kMaxTiles = kSegTiles * kMaxC;
constexpr int kNB = 3;         // segment buffers per CTA
constexpr int kScanW = 3;      // scanner warps per CTA
constexpr int kFinW = 4;       // finalizer warps
constexpr int kWorkW = 9;      // worker warps
constexpr int kNT = 512;
constexpr int kKeys = kMaxC * kScanW;  // one per scanner warp of the cluster
constexpr uint32_t kSat = 1u << 30;
constexpr uint32_t kLimit = 1u << 24;
constexpr uint32_t kExact = 1u << 16;  // meta flag: sum the tile term by term
constexpr uint32_t kCross = 1u << 17;  // meta flag: predicted to cross a binade
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
constexpr float kLog2e = 1.44269504f;
static_assert(kScanW + kFinW + kWorkW == kNT / 32, "warp roles");

// Warp roles: the scanners (warps 0, 4, 8) and a finalizer (12) share warp
// scheduler 0 (warp id mod 4), so the scanners' latency-bound chains never
// compete with the throughput-bound workers for issue slots.
__device__ __forceinline__ int scanner_of(int w) { return (w & 3) == 0 && w < 12 ? w >> 2 : -1; }
__device__ __forceinline__ int finalizer_of(int w) { return w >= 12 ? w - 12 : -1; }
__device__ __forceinline__ int worker_of(int w) { return w - 1 - (w >> 2); }

// Cross-CTA words carry their row: (seq << 32) | payload bits, seq = row + 1
// (0: never written).  A reader polls the word until the seq is the row it
// wants, so the payload needs no separate signal and no fence.
struct Ctl {
    uint64_t sumw[kKeys][kSegTiles];     // this CTA's tile summaries of the row of key k
    uint64_t rowm[kKeys];                // the row max of the row of key k (this CTA's copy)
    uint64_t res[kKeys];                 // the row sum, from the row's scanner
    uint64_t resm[kKeys];                // the row max, from the row's scanner
    uint64_t xm[2][kMaxC];               // segment maxima of rows of parity p
    uint64_t xt[2][kMaxC];               // segment sum estimates
    float tsum[kSegTiles];               // this CTA's tile sum estimates
    uint32_t lmeta[kSegTiles];           // this CTA's predicted binades and flags
    float red[kWorkW];
    __align__(16) float scratch[kScanW][kTileN];  // tile 0 of a scanner's row (float4 reads)
    uint64_t bar_x[kNB];                 // segment landed
    uint64_t bar_sfree[kKeys];           // scanner of that key is done with the summaries
    uint64_t bar_fcred[kScanW];          // C * kFinW arrivals: result slot read everywhere
    int abort_flag;
};

// Members read or written with vector accesses start on their access size.
static_assert(offsetof(Ctl, sumw) % 8 == 0 && offsetof(Ctl, rowm) % 8 == 0 &&
                  offsetof(Ctl, res) % 8 == 0 && offsetof(Ctl, resm) % 8 == 0 &&
                  offsetof(Ctl, xm) % 8 == 0 &&
                  offsetof(Ctl, xt) % 8 == 0, "64-bit words");
static_assert(offsetof(Ctl, scratch) % 16 == 0, "float4 reads of the scratch tile");
static_assert(offsetof(Ctl, bar_x) % 8 == 0 && offsetof(Ctl, bar_sfree) % 8 == 0 &&
                  offsetof(Ctl, bar_fcred) % 8 == 0, "mbarriers");

// ------------------------------------------------------------- cluster PTX
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// Address of this CTA's shared variable p in CTA `cta`'s shared memory.
__device__ __forceinline__ uint32_t remote(const void* p, uint32_t cta) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                 : "=r"(r)
                 : "r"(tbk::smem_addr(p)), "r"(cta));
    return r;
}
// 16-byte loads and stores of this CTA's shared memory by 32-bit shared
// address, so the segment buffers are never reached through generic pointers.
__device__ __forceinline__ float4 lds4(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(a));
    return v;
}
__device__ __forceinline__ void sts4(uint32_t a, const float4& v) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}

// Tagged words: relaxed 64-bit stores and loads at cluster scope (one
// store is seen whole), local or in another CTA of the cluster.
__device__ __forceinline__ uint64_t tag(uint32_t seq, uint32_t payload) {
    return ((uint64_t)seq << 32) | payload;
}
__device__ __forceinline__ void put_word(uint32_t a, uint64_t v) {  // a: cluster address
    asm volatile("st.relaxed.cluster.shared::cluster.u64 [%0], %1;" ::"r"(a), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t get_word(uint32_t a) {  // a: cluster address
    uint64_t v;
    asm volatile("ld.relaxed.cluster.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(a) : "memory");
    return v;
}

// Poll lane-wise words until each active lane's word carries `seq` (each
// lane its own address; inactive lanes pass).  Bounded like every wait: on
// timeout raise the flag, set the abort flag and return what was read.
__device__ __forceinline__ uint64_t poll_word(uint32_t a, bool active, uint32_t seq,
                                              unsigned* status, volatile int* abort_flag) {
    uint64_t v = active ? get_word(a) : 0;
    if (__all_sync(tbk::kFull, !active || (uint32_t)(v >> 32) == seq) || *abort_flag) return v;
    const uint64_t t0 = tbk::global_ns();
    for (;;) {
        if (active) v = get_word(a);
        if (__all_sync(tbk::kFull, !active || (uint32_t)(v >> 32) == seq)) return v;
        if (tbk::global_ns() - t0 > 2000000000ull) {
            if ((threadIdx.x & 31) == 0) atomicOr(status, tbk::kFlagTimeout);
            *abort_flag = 1;
            return v;
        }
    }
}

// A tile summary in one word: D0 (31 bits), D1 - D0 (10 bits, signed), the
// predicted binade (8 bits), kExact, kCross (bits 49, 50), and the row's
// seq modulo 2^13 (bits 51..63).
constexpr int kSeqBits = 13;
__device__ __forceinline__ uint64_t pack_summary(uint2 D, uint32_t mt, uint32_t seq) {
    const int dd = (int)D.y - (int)D.x;
    uint64_t w = (uint64_t)(D.x & 0x7fffffffu);
    w |= (uint64_t)((uint32_t)dd & 0x3ffu) << 31;
    w |= (uint64_t)(mt & 0xffu) << 41;
    w |= (uint64_t)((mt & kExact) ? 1u : 0u) << 49;
    w |= (uint64_t)((mt & kCross) ? 1u : 0u) << 50;
    w |= (uint64_t)(seq & ((1u << kSeqBits) - 1u)) << 51;
    return w;
}
__device__ __forceinline__ uint32_t summary_seq(uint64_t w) { return (uint32_t)(w >> 51); }
__device__ __forceinline__ void unpack_summary(uint64_t w, uint2& D, uint32_t& mt) {
    D.x = (uint32_t)(w & 0x7fffffffu);
    const int dd = ((int)((uint32_t)(w >> 31) & 0x3ffu) << 22) >> 22;
    D.y = (uint32_t)((int)D.x + dd);
    mt = (uint32_t)(w >> 41) & 0xffu;
    if ((w >> 49) & 1u) mt |= kExact;
    if ((w >> 50) & 1u) mt |= kCross;
}

// One arrival on an mbarrier of any CTA of the cluster, ordered after this
// thread's earlier shared-memory stores (release at cluster scope).
__device__ __forceinline__ void arrive_remote(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ bool try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(tbk::smem_addr(bar)), "r"(parity), "r"(tbk::kSuspendHintNs)
        : "memory");
    return done != 0;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Bounded wait on a barrier that remote CTAs arrive on; false (and the CTA
// gives up waiting from then on) after a timeout or an earlier one.
__device__ __forceinline__ bool wait_c(uint64_t* bar, uint32_t parity, unsigned* status,
                                       volatile int* abort_flag) {
    if (*abort_flag) return false;
    if (try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = tbk::global_ns();
    while (!try_wait_cluster(bar, parity)) {
        if (tbk::global_ns() - t0 > 2000000000ull) {
            atomicOr(status, tbk::kFlagTimeout);
            *abort_flag = 1;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void work_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kWorkW * 32) : "memory");
}

// ---------------------------------------------------------------- e and D
// e = 2^fma(x, log2(e), c) with c = rn(-m*log2(e)): one FFMA.  c carries
// an absolute rounding error of up to ulp(m*log2(e))/2, the same for every
// term of the row (a common factor that cancels in e / sum); below
// |m*log2(e)| = 128 it is at most 2^-17.  Rows with a larger max (or no
// finite max) use 2^((x - m)*log2(e)) instead, whose error is relative to
// x - m.
struct Expo {
    float c, m;
    bool slow;
    __device__ __forceinline__ explicit Expo(float mx) : m(mx) {
        c = __fmul_rn(-mx, kLog2e);
        slow = !(fabsf(c) < 128.0f);
    }
    // the row's form, chosen by the caller once per row
    template <bool SLOW>
    __device__ __forceinline__ float at(float x) const {
        const float a = SLOW ? __fmul_rn(__fsub_rn(x, m), kLog2e) : __fmaf_rn(x, kLog2e, c);
        float r;
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
        return r;
    }
    __device__ __forceinline__ float operator()(float x) const {
        return slow ? at<true>(x) : at<false>(x);
    }
};

// Sum over the warp of nonnegative lane values v, to about 2^-21 relative:
// the largest lane value sets a power-of-two scale, each lane rounds
// v * scale to an integer, and one redux.sync adds them (two redux
// instructions instead of a five-step shuffle tree).
__device__ __forceinline__ float warp_sum_est(float v) {
    const uint32_t mx = __reduce_max_sync(tbk::kFull, __float_as_uint(v));  // v >= 0: bits order
    if (mx == 0u) return 0.0f;
    if (mx >= 0x7f800000u) return __uint_as_float(0x7fc00000u);  // inf or NaN
    const int ex = (int)(mx >> 23) - 127;  // the largest lane value is in [2^ex, 2^(ex+1))
    const int sh = 25 - ex;                // lane values < 2^26 after scaling
    if (sh > 126) return 0.0f;             // below 2^-100: no binade anyway
    const float sc = __uint_as_float((uint32_t)(sh + 127) << 23);
    const uint32_t q = __float2uint_rn(__fmul_rn(v, sc));
    const uint32_t tot = __reduce_add_sync(tbk::kFull, q);  // < 32 * 2^26 = 2^31
    return __fmul_rn((float)tot, __uint_as_float((uint32_t)(127 - sh) << 23));
}

__device__ __forceinline__ bool near_pow2(float v) {
    const uint32_t mant = __float_as_uint(v) & 0x7fffffu;
    return mant < (1u << 13) || mant > (1u << 23) - (1u << 13);
}

// Units added by one term given the parity of the partial sum before it.
struct Fn {
    uint32_t a0, a1;  // total for an even / odd running sum at the start
};
__device__ __forceinline__ Fn compose(Fn f, Fn g) {  // f, then g
    Fn r;
    r.a0 = min(f.a0 + ((f.a0 & 1u) ? g.a1 : g.a0), kSat);
    r.a1 = min(f.a1 + (((f.a1 + 1u) & 1u) ? g.a1 : g.a0), kSat);
    return r;
}
__device__ __forceinline__ Fn term_fn(float e, float inv_u) {
    const float a = __fmaf_rn(e, inv_u, kMagic);
    const float r = __fsub_rn(a, kMagic);
    const float d = __fmaf_rn(e, inv_u, -r);
    const uint32_t ri = __float_as_uint(a) - 0x4B400000u;
    if (fabsf(d) != 0.5f) return Fn{ri, ri};
    const uint32_t base = d < 0.0f ? ri - 1u : ri;  // floor(t)
    return Fn{base + (base & 1u), base + ((base + 1u) & 1u)};
}
__device__ __forceinline__ Fn warp_compose(Fn f) {  // lane 0 first; valid in lane 0
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        Fn g;
        g.a0 = __shfl_down_sync(tbk::kFull, f.a0, o);
        g.a1 = __shfl_down_sync(tbk::kFull, f.a1, o);
        if ((lane & (2 * o - 1)) == 0) f = compose(f, g);
    }
    return f;
}


// ------------------------------------------------------------------ scanner
// x of tile `tile` of the row (lane l: terms 8l .. 8l+7; past the row: -inf).
__device__ __forceinline__ void load_tile_x(const float* xr, int tile, int cols, float (&v)[8]) {
    const int lane = threadIdx.x & 31;
    const int n = min(kTileN, cols - tile * kTileN);
    const float* p = xr + (int64_t)tile * kTileN + 8 * lane;
    if (8 * lane + 8 <= n) {
        const float4 a = __ldcg(reinterpret_cast<const float4*>(p));
        const float4 b = __ldcg(reinterpret_cast<const float4*>(p + 4));
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = 8 * lane + k < n ? __ldcg(p + k) : -INFINITY;
    }
}

// Tile `tile` of the row term by term, from its x values.
__device__ __forceinline__ void resolve_tile(tbk::RunSum& st, const float (&xv)[8],
                                             const Expo& ex, int tile, int cols) {
    const int n = min(kTileN, cols - tile * kTileN);
    float e[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) e[k] = ex(xv[k]);
    tbk::ordered_sum_tile<8>(st, e, n, 0);
}

// The in-order sum of the row from the summaries in the cluster's CTAs
// (tile t: CTA t / seg_tiles, slot `key`; lane-uniform result).
__device__ float scan_row(Ctl& ctl, int key, uint32_t seq, int seg_tiles, float* scratch,
                          const float* xr, const Expo& ex, int cols, unsigned* status,
                          volatile int* abort_flag) {
    const int lane = threadIdx.x & 31;
    const int ntiles = (cols + kTileN - 1) / kTileN;
    // tile 0: strictly in order, one lane (four terms per shared load)
    const int n0 = min(cols, kTileN);
    for (int k = lane; k < n0; k += 32) scratch[k] = ex(__ldcg(xr + k));
    __syncwarp();
    float acc = 0.0f;
    if (lane == 0) {
        int k = 0;
        for (; k + 4 <= n0; k += 4) {
            const float4 v = *reinterpret_cast<const float4*>(scratch + k);
            acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, v.x), v.y), v.z), v.w);
        }
        for (; k < n0; ++k) acc = __fadd_rn(acc, scratch[k]);
    }
    acc = __shfl_sync(tbk::kFull, acc, 0);
    __syncwarp();
    tbk::RunSum st;
    st.set(acc);
    for (int t0 = 1; t0 < ntiles && !st.nan; t0 += 32) {
        const int cnt = min(32, ntiles - t0);
        uint2 dl = make_uint2(0u, 0u);
        uint32_t mt = 0;
        {
            const int t = t0 + lane;
            const uint32_t a = lane < cnt ? remote(&ctl.sumw[key][t % seg_tiles],
                                                   (uint32_t)(t / seg_tiles))
                                          : 0u;
            // a summary word is there once it carries this row's seq
            const uint32_t want = seq & ((1u << kSeqBits) - 1u);
            uint64_t w = lane < cnt ? get_word(a) : 0;
            if (!__all_sync(tbk::kFull, lane >= cnt || summary_seq(w) == want) && !*abort_flag) {
                const uint64_t ts = tbk::global_ns();
                for (;;) {
                    if (lane < cnt) w = get_word(a);
                    if (__all_sync(tbk::kFull, lane >= cnt || summary_seq(w) == want)) break;
                    if (tbk::global_ns() - ts > 2000000000ull) {
                        if (lane == 0) atomicOr(status, tbk::kFlagTimeout);
                        *abort_flag = 1;
                        break;
                    }
                }
            }
            if (lane < cnt) unpack_summary(w, dl, mt);
        }
        const int tb = (int)(int8_t)(mt & 0xffu);
        // the first tile predicted to cross: its x is on its way during the scan
        unsigned flagged = __ballot_sync(tbk::kFull, lane < cnt && (mt & kCross));
        int pf = -1;
        float pre[8];
        if (flagged) {
            pf = __ffs(flagged) - 1;
            load_tile_x(xr, t0 + pf, cols, pre);
        }
        int pos = 0;
        while (pos < cnt && !st.nan) {
            const bool valid = lane >= pos && lane < cnt;
            const bool ok = valid && st.fast && !(mt & kExact) && tb == st.b;
            const Fn f = ok ? Fn{dl.x, dl.y} : Fn{0u, 0u};
            Fn inc = f;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                Fn g;
                g.a0 = __shfl_up_sync(tbk::kFull, inc.a0, o);
                g.a1 = __shfl_up_sync(tbk::kFull, inc.a1, o);
                if (lane >= o) inc = compose(g, inc);
            }
            Fn exc;
            exc.a0 = __shfl_up_sync(tbk::kFull, inc.a0, 1);
            exc.a1 = __shfl_up_sync(tbk::kFull, inc.a1, 1);
            if (lane == 0) exc = Fn{0u, 0u};
            const uint32_t p = st.S & 1u;
            const uint32_t exs = p ? exc.a1 : exc.a0;
            const uint32_t mine = ((p + exs) & 1u) ? f.a1 : f.a0;
            const bool ev = valid && (!ok || st.S + exs + mine >= kLimit);
            const unsigned bal = __ballot_sync(tbk::kFull, ev);
            if (bal == 0) {
                st.S += __shfl_sync(tbk::kFull, p ? inc.a1 : inc.a0, 31);
                st.s = __fmul_rn((float)st.S, st.u);
                break;
            }
            const int fl = __ffs(bal) - 1;
            const uint32_t pre_u = __shfl_sync(tbk::kFull, exs, fl);
            if (st.fast && pre_u) {
                st.S += pre_u;
                st.s = __fmul_rn((float)st.S, st.u);
            }
            float xv[8];
            if (fl == pf) {
#pragma unroll
                for (int k = 0; k < 8; ++k) xv[k] = pre[k];
            } else {
                load_tile_x(xr, t0 + fl, cols, xv);
            }
            // the next flagged tile after this one, on its way during the resolve
            flagged &= ~((2u << fl) - 1u);
            if (fl >= pf && flagged) {
                pf = __ffs(flagged) - 1;
                load_tile_x(xr, t0 + pf, cols, pre);
            }
            resolve_tile(st, xv, ex, t0 + fl, cols);
            pos = fl + 1;
        }
    }
    return st.s;
}

// ------------------------------------------------------------------ kernel
__global__ void __launch_bounds__(kNT, 1)
k_softmax_cluster(const float* __restrict__ x, float* y, int rows, int cols, int seg_tiles,
                  unsigned* status) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(16) Ctl ctl;
    float* xbuf = reinterpret_cast<float*>(smem);  // [kNB][seg_tiles * 256]

    uint32_t nc;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(nc));
    const uint32_t me = cluster_rank();
    const int Q = (int)cluster_count(), q = (int)cluster_id();
    const int ncl = (int)nc;
    const int keys = ncl * kScanW;
    const int ntiles = (cols + kTileN - 1) / kTileN;
    const int t0 = (int)me * seg_tiles;                       // first tile of the segment
    const int nt = max(0, min(seg_tiles, ntiles - t0));       // tiles in it
    const int col0 = t0 * kTileN, col1 = min(cols, (t0 + nt) * kTileN);
    const uint32_t seg_bytes = (uint32_t)(col1 - col0) * 4u;
    const int seg_floats = seg_tiles * kTileN;
    const int nloc = rows > q ? (rows - 1 - q) / Q + 1 : 0;   // rows of this cluster
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    volatile int* abort_v = &ctl.abort_flag;

    if (threadIdx.x == 0) {
        for (int b = 0; b < kNB; ++b) tbk::mbar_init(&ctl.bar_x[b], 1);
        for (int k = 0; k < kKeys; ++k) tbk::mbar_init(&ctl.bar_sfree[k], 1);
        for (int s = 0; s < kScanW; ++s) tbk::mbar_init(&ctl.bar_fcred[s], nc * kFinW);
        ctl.abort_flag = 0;
        tbk::fence_mbar_init();
    }
    {  // every tagged word starts with seq 0: never written
        uint64_t* w = &ctl.sumw[0][0];
        const int n = (int)((reinterpret_cast<uint64_t*>(&ctl.tsum) - w));
        for (int i = threadIdx.x; i < n; i += kNT) w[i] = 0;
    }
    __syncthreads();
    cluster_sync_all();  // every CTA's barriers exist before any remote arrive

    const int sw = scanner_of(warp), fw = finalizer_of(warp);
    const int64_t row_stride = cols;
    auto row_of = [&](int j) -> int64_t { return (int64_t)q + (int64_t)j * Q; };

    if (sw >= 0) {
        // ------------------------------------------------------ scanner
        const int key = (int)me + ncl * sw;
        for (int k = 0;; ++k) {
            const int j = key + keys * k;
            if (j >= nloc || *abort_v) break;
            const uint32_t seq = (uint32_t)j + 1u;
            const uint64_t mw = poll_word(tbk::smem_addr(&ctl.rowm[key]), true, seq, status, abort_v);
            const float m = __uint_as_float((uint32_t)mw);
            const Expo ex(m);
            const float* xr = x + row_of(j) * row_stride;
            const float sum =
                scan_row(ctl, key, seq, seg_tiles, ctl.scratch[sw], xr, ex, cols, status, abort_v);
            // the summaries are read: every CTA may write its next row of this key
            __syncwarp();
            if (lane < ncl) arrive_remote(remote(&ctl.bar_sfree[key], (uint32_t)lane));
            // the result slot is free once every finalizer read row j - keys
            if (k >= 1 && !wait_c(&ctl.bar_fcred[sw], (uint32_t)(k - 1) & 1u, status, abort_v))
                break;
            // the result to every CTA: the sum, and the max (the workers'
            // copy of it may already hold a later row when a finalizer looks)
            if (lane < ncl) {
                put_word(remote(&ctl.resm[key], (uint32_t)lane), tag(seq, __float_as_uint(m)));
                put_word(remote(&ctl.res[key], (uint32_t)lane), tag(seq, __float_as_uint(sum)));
            }
        }
    } else if (fw >= 0) {
        // ------------------------------------------------------ finalizers
        const int ft = fw * 32 + lane;
        constexpr int kFin = kFinW * 32;
        constexpr int kU = 16;
        const uint64_t pol = tbk::policy_evict_first();  // last use of x
        const int nv = (col1 - col0) / 4;
        for (int j = 0; j < nloc; ++j) {
            const int key = j % keys;
            const uint32_t seq = (uint32_t)j + 1u;
            const float sum = __uint_as_float(
                (uint32_t)poll_word(tbk::smem_addr(&ctl.res[key]), true, seq, status, abort_v));
            const float m = __uint_as_float(
                (uint32_t)poll_word(tbk::smem_addr(&ctl.resm[key]), true, seq, status, abort_v));
            if (*abort_v) break;
            __syncwarp();
            if (lane == 0)
                arrive_remote(remote(&ctl.bar_fcred[key / ncl], (uint32_t)(key % ncl)));
            const Expo ex(m);
            const bool norm = sum > 0.0f;
            const float inv = __fdiv_rn(1.0f, sum);
            const int64_t base = row_of(j) * row_stride + col0;
            const float4* xr = reinterpret_cast<const float4*>(x + base);
            float4* yr = reinterpret_cast<float4*>(y + base);
            auto run = [&](auto slow_tag) {
                constexpr bool SLOW = decltype(slow_tag)::value;
                auto out = [&](float4 a) {
                    float4 o;
                    o.x = ex.at<SLOW>(a.x); o.y = ex.at<SLOW>(a.y);
                    o.z = ex.at<SLOW>(a.z); o.w = ex.at<SLOW>(a.w);
                    if (norm) {
                        o.x = __fmul_rn(o.x, inv); o.y = __fmul_rn(o.y, inv);
                        o.z = __fmul_rn(o.z, inv); o.w = __fmul_rn(o.w, inv);
                    }
                    return o;
                };
                int v = ft;
                for (; v + (kU - 1) * kFin < nv; v += kU * kFin) {
                    float4 a[kU];
#pragma unroll
                    for (int u = 0; u < kU; ++u) a[u] = tbk::ld_f4_hint(xr + v + u * kFin, pol);
#pragma unroll
                    for (int u = 0; u < kU; ++u) __stcs(yr + v + u * kFin, out(a[u]));
                }
                for (; v < nv; v += kFin) __stcs(yr + v, out(tbk::ld_f4_hint(xr + v, pol)));
            };
            if (ex.slow)
                run(std::true_type{});
            else
                run(std::false_type{});
        }
    } else {
        // ------------------------------------------------------ workers
        const int wi = worker_of(warp);
        const bool producer = wi == 0 && lane == 0;
        const uint64_t pol_keep = tbk::policy_evict_last();  // the finalizers read x again
        auto seg = [&](int b) { return xbuf + (size_t)b * seg_floats; };
        const uint32_t xbuf_s = tbk::smem_addr(xbuf);
        // shared address of term 0 of tile t of buffer b
        auto tile_s = [&](int b, int t) {
            return xbuf_s + (uint32_t)(b * seg_floats + t * kTileN) * 4u;
        };
        auto issue = [&](int j) {  // one thread: row j's segment into buffer j % kNB
            const int b = j % kNB;
            tbk::mbar_expect_tx(&ctl.bar_x[b], seg_bytes);
            if (seg_bytes)
                tbk::bulk_g2s_hint(seg(b), x + row_of(j) * row_stride + col0, seg_bytes,
                                   &ctl.bar_x[b], pol_keep);
        };
        int issued = 0;  // rows whose copy was issued
        if (producer)
            for (; issued < min(kNB, nloc); ++issued) issue(issued);
        const int nfull = (col1 - col0) / kTileN;  // full tiles of the segment
        // lane l holds terms 4l..4l+3 and 128+4l..128+4l+3 of a tile
        auto ld2 = [&](uint32_t ts, int t, float4& a, float4& c) {
            if (t < nfull) {
                a = lds4(ts + 16u * lane);
                c = lds4(ts + 512u + 16u * lane);
            } else {  // the row's ragged last tile (a multiple of 4 terms)
                const int n = (col1 - col0) - t * kTileN;
                a = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
                c = a;
                if (4 * lane < n) a = lds4(ts + 16u * lane);
                if (128 + 4 * lane < n) c = lds4(ts + 512u + 16u * lane);
            }
        };
        auto st2 = [&](uint32_t ts, int t, const float4& a, const float4& c) {
            const int n = t < nfull ? kTileN : (col1 - col0) - t * kTileN;
            if (4 * lane < n) sts4(ts + 16u * lane, a);
            if (128 + 4 * lane < n) sts4(ts + 512u + 16u * lane, c);
        };

        // Phase A: segment max -> every CTA.
        auto phase_a = [&](int j) {
            const int b = j % kNB;
            wait_c(&ctl.bar_x[b], (uint32_t)(j / kNB) & 1u, status, abort_v);
            float mx = -INFINITY, my = -INFINITY;
            for (int t = wi; t < nt; t += 2 * kWorkW) {
                const int u = t + kWorkW;
                float4 a, c, a2, c2;
                ld2(tile_s(b, t), t, a, c);
                if (u < nt) ld2(tile_s(b, u), u, a2, c2);
                mx = fmaxf(mx, fmaxf(fmaxf(fmaxf(a.x, a.y), fmaxf(a.z, a.w)),
                                     fmaxf(fmaxf(c.x, c.y), fmaxf(c.z, c.w))));
                if (u < nt)
                    my = fmaxf(my, fmaxf(fmaxf(fmaxf(a2.x, a2.y), fmaxf(a2.z, a2.w)),
                                         fmaxf(fmaxf(c2.x, c2.y), fmaxf(c2.z, c2.w))));
            }
            mx = tbk::warp_max(fmaxf(mx, my));
            if (lane == 0) ctl.red[wi] = mx;
            work_sync();
            if (wi == 0) {
                float mc = ctl.red[0];
#pragma unroll
                for (int w = 1; w < kWorkW; ++w) mc = fmaxf(mc, ctl.red[w]);
                if (lane < ncl)
                    put_word(remote(&ctl.xm[j & 1][me], (uint32_t)lane),
                             tag((uint32_t)j + 1u, __float_as_uint(mc)));
            }
        };
        // Phase B: e in place, tile estimates, segment estimate -> every CTA.
        auto phase_b = [&](int j) -> float {
            // every warp reads the cluster's segment maxima itself (lane c: CTA c's)
            const uint64_t mw = poll_word(tbk::smem_addr(&ctl.xm[j & 1][lane & (kMaxC - 1)]),
                                          lane < ncl, (uint32_t)j + 1u, status, abort_v);
            const float m = tbk::warp_max(lane < ncl ? __uint_as_float((uint32_t)mw) : -INFINITY);
            const Expo ex(m);
            const int b = j % kNB;
            auto run = [&](auto slow_tag) {
                constexpr bool SLOW = decltype(slow_tag)::value;
                auto e4 = [&](float4& v) {
                    v.x = ex.at<SLOW>(v.x); v.y = ex.at<SLOW>(v.y);
                    v.z = ex.at<SLOW>(v.z); v.w = ex.at<SLOW>(v.w);
                };
                for (int t = wi; t < nt; t += 2 * kWorkW) {
                    const int u = t + kWorkW;
                    float4 a, c, a2, c2;
                    ld2(tile_s(b, t), t, a, c);
                    if (u < nt) ld2(tile_s(b, u), u, a2, c2);
                    e4(a); e4(c);
                    if (u < nt) {
                        e4(a2); e4(c2);
                    }
                    st2(tile_s(b, t), t, a, c);
                    if (u < nt) st2(tile_s(b, u), u, a2, c2);
                    const float s1 = warp_sum_est(((a.x + a.y) + (a.z + a.w)) +
                                                  ((c.x + c.y) + (c.z + c.w)));
                    if (lane == 0) ctl.tsum[t] = s1;
                    if (u < nt) {
                        const float s2 = warp_sum_est(((a2.x + a2.y) + (a2.z + a2.w)) +
                                                      ((c2.x + c2.y) + (c2.z + c2.w)));
                        if (lane == 0) ctl.tsum[u] = s2;
                    }
                }
            };
            if (ex.slow)
                run(std::true_type{});
            else
                run(std::false_type{});
            work_sync();
            if (wi == 0) {
                float v = 0.0f;
                for (int t = lane; t < nt; t += 32) v += ctl.tsum[t];
                v = tbk::warp_sum(v);
                if (lane < ncl)
                    put_word(remote(&ctl.xt[j & 1][me], (uint32_t)lane),
                             tag((uint32_t)j + 1u, __float_as_uint(v)));
            }
            return m;
        };
        // Phase C: predicted binades, (D0, D1) per tile -> this CTA's summary
        // slot of the row's key; one arrive tells the row's scanner.
        auto phase_c = [&](int j, float m) {
            const int key = j % keys;
            const uint32_t seq = (uint32_t)j + 1u;
            if (wi == 0) {
                // the segments' sum estimates; the running sum at this
                // segment's start is the sum of those before it
                const uint64_t tw = poll_word(tbk::smem_addr(&ctl.xt[j & 1][lane & (kMaxC - 1)]),
                                              lane < ncl, seq, status, abort_v);
                float run = 0.0f;
                for (int c = 0; c < (int)me; ++c)
                    run += __uint_as_float((uint32_t)__shfl_sync(tbk::kFull, (uint32_t)tw, c));
                // warp scan of the segment's tile estimates (two per lane)
                const float v0 = 2 * lane < nt ? ctl.tsum[2 * lane] : 0.0f;
                const float v1 = 2 * lane + 1 < nt ? ctl.tsum[2 * lane + 1] : 0.0f;
                float inc = v0 + v1;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const float nb = __shfl_up_sync(tbk::kFull, inc, o);
                    if (lane >= o) inc += nb;
                }
                float ex0 = __shfl_up_sync(tbk::kFull, inc, 1);
                if (lane == 0) ex0 = 0.0f;
                const float p0 = run + ex0, p1 = p0 + v0, p2 = p1 + v1;
                auto meta_of = [](float a, float b) {
                    const int ba = tbk::binade_of(a);
                    uint32_t f = (uint32_t)ba & 0xffu;
                    if (ba == tbk::kNoBinade) f |= kExact;
                    if (tbk::binade_of(b) != ba || near_pow2(a) || near_pow2(b)) f |= kCross;
                    return f;
                };
                if (2 * lane < nt) ctl.lmeta[2 * lane] = meta_of(p0, p1);
                if (2 * lane + 1 < nt) ctl.lmeta[2 * lane + 1] = meta_of(p1, p2);
            }
            // the scanner of this key must be done with row j - keys
            if (j >= keys)
                wait_c(&ctl.bar_sfree[key], (uint32_t)(j / keys - 1) & 1u, status, abort_v);
            work_sync();
            const int b = j % kNB;
            auto units = [&](int t, const float4& a, const float4& c, bool& big, bool& tie,
                             float& iu_out) -> uint32_t {
                const uint32_t mt = ctl.lmeta[t];
                const float iu = tbk::inv_grid((int)(int8_t)(mt & 0xffu));
                iu_out = iu;
                const float e[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
                // Every term below 2^22 grid units makes the magic rounding
                // exact: certain when the tile's estimate is below 2^21
                // units, checked term by term otherwise.
                const bool small = __fmul_rn(ctl.tsum[t], iu) < 2097152.0f;
                uint32_t acc = 0;
                float dm = 0.0f;
                bool bad = false;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float fa = __fmaf_rn(e[k], iu, kMagic);
                    acc += __float_as_uint(fa);
                    const float r = __fsub_rn(fa, kMagic);
                    dm = fmaxf(dm, fabsf(__fmaf_rn(e[k], iu, -r)));
                    if (!small) bad |= !(fa < 16777216.0f);  // t >= 2^22, or NaN
                }
                big = !small && __any_sync(tbk::kFull, bad);
                tie = __any_sync(tbk::kFull, dm == 0.5f);
                return __reduce_add_sync(tbk::kFull, acc - 8u * 0x4B400000u);
            };
            auto finish = [&](int t, const float4& a, const float4& c, uint32_t sum_u, bool big,
                              bool tie, float iu) {
                const uint32_t mt = ctl.lmeta[t];
                uint2 D = make_uint2(sum_u, sum_u);
                if (mt & kExact) {
                    D = make_uint2(0u, 0u);
                } else if (big) {
                    D = make_uint2(kSat, kSat);
                } else if (tie) {
                    const float e[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
                    Fn fa{0u, 0u}, fb{0u, 0u};
#pragma unroll
                    for (int k = 0; k < 4; ++k) fa = compose(fa, term_fn(e[k], iu));
#pragma unroll
                    for (int k = 4; k < 8; ++k) fb = compose(fb, term_fn(e[k], iu));
                    fa = warp_compose(fa);
                    fb = warp_compose(fb);
                    const Fn ft = compose(fa, fb);
                    D = make_uint2(ft.a0, ft.a1);
                }
                const int dd = (int)D.y - (int)D.x;
                uint32_t mw = mt;
                if (dd < -512 || dd > 511) {  // cannot be packed: term by term
                    D = make_uint2(0u, 0u);
                    mw |= kExact;
                }
                if (lane == 0)
                    put_word(tbk::smem_addr(&ctl.sumw[key][t]), pack_summary(D, mw, seq));
            };
            for (int t = wi; t < nt; t += 2 * kWorkW) {
                const int u = t + kWorkW;
                float4 a, c, a2, c2;
                ld2(tile_s(b, t), t, a, c);
                if (u < nt) ld2(tile_s(b, u), u, a2, c2);
                // terms past the row are -inf before the exp pass and 0 after it
                if (t >= nfull) {
                    const int n = (col1 - col0) - t * kTileN;
                    if (4 * lane >= n) a = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (128 + 4 * lane >= n) c = make_float4(0.f, 0.f, 0.f, 0.f);
                }
                if (u < nt && u >= nfull) {
                    const int n = (col1 - col0) - u * kTileN;
                    if (4 * lane >= n) a2 = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (128 + 4 * lane >= n) c2 = make_float4(0.f, 0.f, 0.f, 0.f);
                }
                bool big1, tie1, big2 = false, tie2 = false;
                float iu1, iu2 = 0.0f;
                const uint32_t s1 = units(t, a, c, big1, tie1, iu1);
                uint32_t s2 = 0;
                if (u < nt) s2 = units(u, a2, c2, big2, tie2, iu2);
                finish(t, a, c, s1, big1, tie1, iu1);
                if (u < nt) finish(u, a2, c2, s2, big2, tie2, iu2);
            }
            // the row max for this CTA's scanner and finalizers
            if (wi == 0 && lane == 0)
                put_word(tbk::smem_addr(&ctl.rowm[key]), tag(seq, __float_as_uint(m)));
            work_sync();
            // the buffer is free: the row kNB ahead is copied into it
            if (producer && issued < nloc && !*abort_v) {
                tbk::fence_proxy_async_shared();
                issue(issued);
                ++issued;
            }
        };

        if (nloc > 0) phase_a(0);
        for (int j = 0; j < nloc; ++j) {
            const float m = phase_b(j);
            if (j + 1 < nloc) phase_a(j + 1);
            phase_c(j, m);
        }
        // No copy may still be writing this CTA's shared memory at exit
        // (possible only after a timeout): a last bounded wait on each.
        if (producer)
            for (int r = max(0, issued - kNB); r < issued; ++r)
                tbk::mbar_wait(&ctl.bar_x[r % kNB], (uint32_t)(r / kNB) & 1u, status, 200000000ull);
    }
    __syncwarp();
    __syncthreads();
    cluster_sync_all();  // no CTA leaves while a peer may still write its shared memory
}

}  // namespace

namespace tbh {

bool softmax_use_cluster() {
    const char* e = getenv("TB_B200_SOFTMAX");
    return e && !strcmp(e, "cluster");
}

// f32 softmax through k_softmax_cluster.  Returns 1 (nothing launched) when
// the shape is not one it handles: fewer than 1024 or more than 131072
// columns, a column count that is not a multiple of 4, or unaligned rows.
int softmax_cluster_f32(int64_t rows, int64_t cols, const float* x, float* y, cudaStream_t s) {
    if (cols < 1024 || cols > (int64_t)kMaxTiles * kTileN || cols % 4 || !aligned16(x) ||
        !aligned16(y) || rows > INT32_MAX)
        return 1;
    DeviceState* ds = current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    const int ntiles = (int)((cols + kTileN - 1) / kTileN);
    const int C = (ntiles + kSegTiles - 1) / kSegTiles;
    const int seg_tiles = (ntiles + C - 1) / C;
    const size_t smem = (size_t)kNB * seg_tiles * kTileN * sizeof(float);
    static thread_local size_t attr_set[64];
    static thread_local int clusters_cache[64][kMaxC + 1];
    const int dv = ds->device;
    if (dv < 0 || dv >= 64) return 1;
    if (attr_set[dv] < smem) {
        TB_CUDA_TRY(cudaFuncSetAttribute(k_softmax_cluster,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr_set[dv] = smem;
        for (int c = 0; c <= kMaxC; ++c) clusters_cache[dv][c] = 0;
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.blockDim = dim3(kNT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    int& Q = clusters_cache[dv][C];
    if (Q == 0) {
        cfg.gridDim = dim3((unsigned)(C * ds->sm_count));
        int n = 0;
        TB_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, k_softmax_cluster, &cfg));
        if (n < 1) return 1;
        Q = n;
    }
    const int nclu = (int)(rows < Q ? rows : Q);
    cfg.gridDim = dim3((unsigned)(nclu * C));
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_softmax_cluster, static_cast<const float*>(x),
                                             y, (int)rows, (int)cols, seg_tiles, ds->status);
    count_launch();
    if (e != cudaSuccess) {
        set_error("softmax kernel (cluster)", e);
        return TB_ERR_DEVICE;
    }
    return TB_OK;
}

}  // namespace tbh
