// k_softmax_staged.cu -- f32 row softmax for rows of up to 32768 terms:
// each row's exponentials staged once in shared memory, the reference's
// in-order sum scanned by dedicated warps while the next rows go on.
//
// Reference arithmetic (tb_cpu_softmax_f32, src/ops/softmax.c:4-32):
//   m = max x (strict '>', from -inf);  e_i = expf(x_i - m);
//   sum = ((e_0 + e_1) + e_2) + ...  (f32, in order);  y_i = e_i * (1.0f/sum) if sum > 0.
// e here is __expf(x - m) (ex2-based; at most 2 + 1.173|x - m| ulp from exp,
// which weighted by e itself stays below 4e-7 of the largest term), computed
// by one expression everywhere so every pass sees the same bits.  The sum is
// the in-order f32 sum of those terms, bit for bit (see ordered_sum.cuh for
// the integer-grid argument).
//
// CTA = 24 warps, persistent over rows blockIdx.x, +gridDim.x, ... (one CTA
// per SM at V = 32000: the row buffer is 125 KB of shared memory):
//   warps 0,4,8 scanners: the ordered sum of every third row, from the tile
//               summaries below (three summary buffers), while the workers
//               go on.  They share one warp scheduler.
//   6 warps     finalizers: y = e * (1/sum) of each scanned row, e recomputed
//               from x (still in L2), streaming stores.
//   15 warps    workers, per row (the row is prefetched to L2 one row
//               ahead, so HBM is read once):
//     exp    e = ex2(...) from x in L2 into the row buffer, and a sum
//            estimate per 256-term tile.
//     est    running-sum estimate at each tile start -> predicted binade b_t;
//            tiles likely to cross a binade (or near a power of two) get a
//            slot: a copy of their terms for the scanner.  Beside it, one
//            warp sums tile 0 in order and 13 warps take the next row's max
//            from L2, so no row waits for its max.
//     units  per tile, the integer sum of rne(e / u_b) as a function of the
//            running sum's parity at the tile start: (D0, D1).  Only exact
//            ties (e/u = k + 1/2) make them differ; round-to-even then
//            depends on the parity of the partial sum.
//     handoff the summaries go to the row's scanner.
//   The scanner walks 32 tiles per step: an ordered composition scan of the
//   (D0, D1) functions gives every tile's exact start offset; the first tile
//   that is not in the current binade, is flagged, or crosses 2^24 units is
//   resolved -- in a slotted tile by prefix sums of its grid units and a
//   ballot (the crossing term is one real f32 addition, the rest of the tile
//   O(1) on the next grid), otherwise term by term (ordered_sum_tile).
// Every wait is bounded (tma.cuh); a timeout raises TB_B200_FLAG_WAIT_TIMEOUT,
// after which the CTA skips its remaining waits and ends.  (An earlier form
// copied each row into shared memory with bulk copies: the copy of the next
// row could only start once the buffer was free, and its landing was on
// every row's critical path.)
#include <math.h>

#include "ordered_sum.cuh"
#include "tb_device.cuh"
#include "tb_internal.h"
#include "tma.cuh"
#include "scan_tiles.cuh"

namespace {

using namespace tbsm;

constexpr int kNT = 768;
constexpr int kScanWarps = 3;
constexpr int kBufs = kScanWarps;  // summary/slot buffers: row i uses i % kBufs
constexpr int kFinWarps = 6;  // finalizers: the normalising pass, beside the workers
constexpr int kFin = kFinWarps * 32;
constexpr int kWorkWarps = kNT / 32 - kScanWarps - kFinWarps;
constexpr int kWork = kWorkWarps * 32;
constexpr int kMaxCols = 32768;
constexpr int kMaxTiles = kMaxCols / kTileN;
constexpr int kMaxSlots = 16;
constexpr uint64_t kStaggerNs = 7000;  // start offset of odd CTAs

// Hand-off from the workers to a row's scanner (double-buffered).
struct RowSummary {
    uint2 D[kMaxTiles];        // (D0, D1) per tile
    uint32_t meta[kMaxTiles];  // predicted binade (int8) | kExact | slot << 24
    float m;                   // the row max
    float s0;                  // in-order sum of tile 0's terms
    float pad[2];
};

__device__ __forceinline__ void work_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(kWork) : "memory");
}

struct Shared {
    float* xbuf;
    RowSummary* sum;  // [2]
    float* tsum;      // [kMaxTiles]
    Slot* slots;      // [2][nslot]
};

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, unsigned* status,
                                         volatile int* abort_flag) {
    if (*abort_flag) return false;
    if (tbk::mbar_wait(bar, parity, status)) return true;
    *abort_flag = 1;
    return false;
}

// ------------------------------------------------------------------ scanner
// Terms of a tile that has no slot, recomputed from x (still in L2).
struct XTerms {
    const float* xr;
    float m;
    __device__ __forceinline__ void operator()(int tile, int n, float (&e)[8]) const {
        const int lane = threadIdx.x & 31;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int j = lane * 8 + k;
            e[k] = j < n ? expo(xr[(int64_t)tile * kTileN + j], m) : 0.0f;
        }
    }
};

// ------------------------------------------------------------------ kernel
__global__ void __launch_bounds__(kNT, 1)
k_softmax_staged(const float* x, float* y, int rows, int cols, int nslot, unsigned* status) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bar_ready[kBufs], bar_done[kBufs];
    __shared__ float red[kWorkWarps];      // the next row's max, per worker warp
    __shared__ float row_sum[4];           // ordered sum of row i at i & 3 (scanner -> finalizers)
    __shared__ float row_m[4];             // row max of row i at i & 3 (workers -> finalizers)
    __shared__ __align__(8) uint64_t bar_fin[4];  // finalizers have read row_sum/row_m of row i
    __shared__ int abort_flag;

    const int ntiles = (cols + kTileN - 1) / kTileN;
    Shared sh;
    sh.xbuf = reinterpret_cast<float*>(smem);  // the row buffer
    sh.sum = reinterpret_cast<RowSummary*>(smem + (size_t)ntiles * kTileN * 4);
    sh.tsum = reinterpret_cast<float*>(sh.sum + kBufs);
    sh.slots = reinterpret_cast<Slot*>(sh.tsum + kMaxTiles);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nloc = rows > (int)blockIdx.x ? (rows - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const uint32_t rowbytes = (uint32_t)cols * 4u;
    volatile int* abort_v = &abort_flag;

    if (threadIdx.x == 0) {
        for (int k = 0; k < kBufs; ++k) {
            tbk::mbar_init(&bar_ready[k], 1);
            tbk::mbar_init(&bar_done[k], 1);
        }
        for (int k = 0; k < 4; ++k) tbk::mbar_init(&bar_fin[k], kFin);
        abort_flag = 0;
        tbk::fence_mbar_init();
    }
    __syncthreads();

    // Scanners are warps 0, 4, 8: one warp scheduler (warp id mod 4) runs
    // them beside a single worker warp, so their latency-bound chains are
    // not starved of issue slots by the throughput-bound workers.
    const bool scanner = (warp & 3) == 0 && (warp >> 2) < kScanWarps;
    if (scanner) {
        // ---------------- scanner sc takes rows sc, sc + kBufs, ...
        const int sc = warp >> 2;
        for (int i = sc; i < nloc; i += kScanWarps) {
            wait_bar(&bar_ready[sc], (uint32_t)(i / kBufs) & 1u, status, abort_v);
            const int row = (int)blockIdx.x + i * (int)gridDim.x;
            const RowSummary& R = sh.sum[sc];
            const float sum = scan_tiles(R.D, R.meta, R.s0, sh.slots + sc * nslot, nslot,
                                         XTerms{x + (int64_t)row * cols, R.m}, cols);
            if (lane == 0) row_sum[i & 3] = sum;
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();
                tbk::mbar_arrive(&bar_done[sc]);
            }
        }
        return;
    }

    const int nw = warp - min(kScanWarps, (warp + 3) >> 2);  // index among the other warps
    if (nw < kFinWarps) {
        // ---------------- finalizers: y = e * (1/sum) of each row once it is
        //                  scanned, x re-read from L2, while the workers
        //                  process the following rows
        const int ft = nw * 32 + lane;
        const uint64_t pol = tbk::policy_evict_first();  // last use of x
        for (int i = 0; i < nloc; ++i) {
            wait_bar(&bar_done[i % kBufs], (uint32_t)(i / kBufs) & 1u, status, abort_v);
            const float sum = row_sum[i & 3];
            const float mp = row_m[i & 3];
            tbk::mbar_arrive(&bar_fin[i & 3]);  // this thread is done with slot i & 3
            const bool norm = sum > 0.0f;
            const float inv = __fdiv_rn(1.0f, sum);
            const int64_t row = (int64_t)blockIdx.x + (int64_t)i * gridDim.x;
            const float4* xr = reinterpret_cast<const float4*>(x + row * cols);
            float4* yr = reinterpret_cast<float4*>(y + row * cols);
            const int nv = cols / 4;
            constexpr int kU = 12;
            int v = ft;
            for (; v + (kU - 1) * kFin < nv; v += kU * kFin) {
                float4 q[kU];
#pragma unroll
                for (int u = 0; u < kU; ++u) q[u] = tbk::ld_f4_hint(xr + v + u * kFin, pol);
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    float4 o;
                    o.x = expo(q[u].x, mp); o.y = expo(q[u].y, mp);
                    o.z = expo(q[u].z, mp); o.w = expo(q[u].w, mp);
                    if (norm) {
                        o.x = __fmul_rn(o.x, inv); o.y = __fmul_rn(o.y, inv);
                        o.z = __fmul_rn(o.z, inv); o.w = __fmul_rn(o.w, inv);
                    }
                    __stcs(yr + v + u * kFin, o);
                }
            }
            for (; v < nv; v += kFin) {
                const float4 q = tbk::ld_f4_hint(xr + v, pol);
                float4 o;
                o.x = expo(q.x, mp); o.y = expo(q.y, mp); o.z = expo(q.z, mp); o.w = expo(q.w, mp);
                if (norm) {
                    o.x = __fmul_rn(o.x, inv); o.y = __fmul_rn(o.y, inv);
                    o.z = __fmul_rn(o.z, inv); o.w = __fmul_rn(o.w, inv);
                }
                __stcs(yr + v, o);
            }
        }
        return;
    }

    // ---------------- workers
    // Odd CTAs start half a row period later: the CTAs alternate between
    // their memory-bound and compute-bound phases instead of all hitting
    // HBM at once.
    if (blockIdx.x & 1) {
        const uint64_t t0 = tbk::global_ns();
        while (tbk::global_ns() - t0 < kStaggerNs) {
        }
    }
    const int ww = nw - kFinWarps;  // worker index 0..kWorkWarps-1
    const int wt = ww * 32 + lane;
    const uint64_t pol_last = tbk::policy_evict_last();
    const int nfull = cols / kTileN;
    auto row_x = [&](int i) { return x + ((int64_t)blockIdx.x + (int64_t)i * gridDim.x) * cols; };
    // The max of a row, read from global memory (L2), over the tiles of
    // worker warps w0 .. w0 + nwk - 1: the warp's part, into red[ww].
    // Four tiles' loads are in flight per lane before their maxima.
    auto part_max = [&](const float* xr, int w0, int nwk) {
        constexpr int kU = 4;
        float mx = -INFINITY;
        if (ww >= w0 && ww < w0 + nwk) {
            for (int t = ww - w0; t < ntiles; t += kU * nwk) {
                float4 v[2 * kU];
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    const int tu = t + u * nwk;
                    const float* xt = xr + (int64_t)tu * kTileN;
                    const int n = tu < ntiles ? min(kTileN, cols - tu * kTileN) : 0;
                    v[2 * u] = v[2 * u + 1] = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
                    if (4 * lane < n) v[2 * u] = *reinterpret_cast<const float4*>(xt + 4 * lane);
                    if (128 + 4 * lane < n)
                        v[2 * u + 1] = *reinterpret_cast<const float4*>(xt + 128 + 4 * lane);
                }
#pragma unroll
                for (int q = 0; q < 2 * kU; ++q)
                    mx = fmaxf(mx, fmaxf(fmaxf(v[q].x, v[q].y), fmaxf(v[q].z, v[q].w)));
            }
            mx = tbk::warp_max(mx);
        }
        if (lane == 0) red[ww] = mx;
    };
    if (nloc > 0) {  // row 0's max, by every worker
        if (wt == 0) tbk::prefetch_l2_hint(row_x(0), rowbytes, pol_last);
        part_max(row_x(0), 0, kWorkWarps);
        work_sync();
    }
    for (int i = 0; i < nloc; ++i) {
        // The next row heads for L2 while this one is worked on: its max is
        // read during this row's estimate, its terms at the start of the next.
        if (wt == 0 && i + 1 < nloc && !*abort_v)
            tbk::prefetch_l2_hint(row_x(i + 1), rowbytes, pol_last);
        auto tp = [&](int t) -> float* { return sh.xbuf + (size_t)t * kTileN; };
        {
            const int k = i % kBufs;
            RowSummary& R = sh.sum[k];
            Slot* SL = sh.slots + k * nslot;
            float m = red[0];
#pragma unroll
            for (int w = 1; w < kWorkWarps; ++w) m = fmaxf(m, red[w]);
            // ---- e into the row buffer, from x in L2, + tile sums (full tiles
            //      unconditional; the last tile may be partial)
            const float* xr = row_x(i);
            for (int t0 = ww; t0 < ntiles; t0 += 2 * kWorkWarps) {
                float4 v[4];  // two tiles' loads in flight per lane
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int t = t0 + u * kWorkWarps;
                    const float* gt = xr + (int64_t)t * kTileN;
                    const int n = t < ntiles ? min(kTileN, cols - t * kTileN) : 0;
                    v[2 * u] = v[2 * u + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (4 * lane < n) v[2 * u] = *reinterpret_cast<const float4*>(gt + 4 * lane);
                    if (128 + 4 * lane < n)
                        v[2 * u + 1] = *reinterpret_cast<const float4*>(gt + 128 + 4 * lane);
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int t = t0 + u * kWorkWarps;
                    if (t >= ntiles) break;  // warp-uniform
                    const int n = min(kTileN, cols - t * kTileN);
                    float* xt = tp(t);
                    float4 a = v[2 * u], b = v[2 * u + 1];
                    a.x = expo(a.x, m); a.y = expo(a.y, m); a.z = expo(a.z, m); a.w = expo(a.w, m);
                    b.x = expo(b.x, m); b.y = expo(b.y, m); b.z = expo(b.z, m); b.w = expo(b.w, m);
                    float s = 0.0f;
                    if (4 * lane < n) {
                        *reinterpret_cast<float4*>(xt + 4 * lane) = a;
                        s = (a.x + a.y) + (a.z + a.w);
                    }
                    if (128 + 4 * lane < n) {
                        *reinterpret_cast<float4*>(xt + 128 + 4 * lane) = b;
                        s += (b.x + b.y) + (b.z + b.w);
                    }
                    s = warp_sum_est(s);
                    if (lane == 0) sh.tsum[t] = s;
                }
            }
            // Buffer k last held row i - kBufs: its scan must be over.  The
            // finalizers must have taken row i-3's sum and max: then ring slot
            // i & 3 (row i-4) is free, and no scanner completes a phase of its
            // done barrier (row i's, once handed off) before the finalizers have
            // waited on the one before -- each barrier stays at most one phase
            // ahead of its waiters.
            if (i >= kBufs)
                wait_bar(&bar_done[k], (uint32_t)((i - kBufs) / kBufs) & 1u, status, abort_v);
            if (i >= 3) wait_bar(&bar_fin[(i - 3) & 3], (uint32_t)((i - 3) >> 2) & 1u, status, abort_v);
            work_sync();
            // ---- tile 0's in-order sum, by the last worker warp, beside the
            //      estimate below (the row buffer still holds e)
            if (ww == kWorkWarps - 1 && lane == 0) {
                const int n0 = min(cols, kTileN);
                const float* e0 = tp(0);
                float acc = 0.0f;
                if (n0 == kTileN) {
#pragma unroll 16
                    for (int q = 0; q < kTileN; q += 4) {
                        const float4 v = *reinterpret_cast<const float4*>(e0 + q);
                        acc = __fadd_rn(acc, v.x);
                        acc = __fadd_rn(acc, v.y);
                        acc = __fadd_rn(acc, v.z);
                        acc = __fadd_rn(acc, v.w);
                    }
                } else {
                    for (int q = 0; q < n0; ++q) acc = __fadd_rn(acc, e0[q]);
                }
                R.s0 = acc;
            }
            // ---- estimate -> predicted binades, slots (first worker warp)
            if (ww == 0) {
                float v[4];
                float local = 0.0f;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int t = 4 * lane + q;
                    v[q] = t < ntiles ? sh.tsum[t] : 0.0f;
                    local += v[q];
                }
                float inc = local;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const float nb = __shfl_up_sync(tbk::kFull, inc, o);
                    if (lane >= o) inc += nb;
                }
                float run = __shfl_up_sync(tbk::kFull, inc, 1);
                if (lane == 0) run = 0.0f;
                int bq[4];
                unsigned lk = 0;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int t = 4 * lane + q;
                    const int b = tbk::binade_of(run);
                    const float nxt = run + v[q];
                    bq[q] = b;
                    if (t < ntiles && (t == 0 || b == tbk::kNoBinade || tbk::binade_of(nxt) != b ||
                                       near_pow2(run) || near_pow2(nxt)))
                        lk |= 1u << q;
                    run = nxt;
                }
                const uint32_t cnt = __popc(lk);
                uint32_t sl = warp_incl(cnt) - cnt;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int t = 4 * lane + q;
                    if (t >= ntiles) continue;
                    uint32_t slot = kNoSlot;
                    if ((lk >> q) & 1u) {
                        if (sl < (uint32_t)nslot) slot = sl;
                        ++sl;
                    }
                    R.meta[t] = ((uint32_t)bq[q] & 0xffu) | (slot << 24);
                }
                if (lane == 0) {
                    R.m = m;
                    row_m[i & 3] = m;
                }
            }
            // ---- the next row's max, from L2, by the workers the estimate and
            //      tile 0 leave free (warps 1 .. kWorkWarps - 2)
            if (i + 1 < nloc)
                part_max(row_x(i + 1), 1, kWorkWarps - 2);
            work_sync();
            // ---- units: (D0, D1) per tile; a slotted tile's terms go to its slot
            {
                for (int t = ww; t < ntiles; t += kWorkWarps) {
                    const float* xt = tp(t);
                    const uint32_t meta = R.meta[t];
                    const int b = (int)(int8_t)(meta & 0xffu);
                    const uint32_t slot = meta >> 24;
                    float4 a, c;
                    if (t < nfull) {
                        a = *reinterpret_cast<const float4*>(xt + 4 * lane);
                        c = *reinterpret_cast<const float4*>(xt + 128 + 4 * lane);
                    } else {
                        const int n = cols - t * kTileN;
                        a = make_float4(0.f, 0.f, 0.f, 0.f);
                        c = a;
                        if (4 * lane < n) a = *reinterpret_cast<const float4*>(xt + 4 * lane);
                        if (128 + 4 * lane < n) c = *reinterpret_cast<const float4*>(xt + 128 + 4 * lane);
                    }
                    if (slot < (uint32_t)nslot) {  // warp-uniform; terms past cols are 0
                        Slot& S = SL[slot];
                        *reinterpret_cast<float4*>(S.e + 4 * lane) = a;
                        *reinterpret_cast<float4*>(S.e + 128 + 4 * lane) = c;
                    }
                    const float e[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
                    const float iu = tbk::inv_grid(b == tbk::kNoBinade ? 0 : b);
                    float acc = 0.0f, dm = 0.0f;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float tt = __fmul_rn(e[q], iu);
                        const float r = __fsub_rn(__fadd_rn(tt, kMagic), kMagic);
                        acc = __fadd_rn(acc, r);
                        dm = fmaxf(dm, fabsf(__fsub_rn(tt, r)));
                    }
                    // acc < 2^22 - 1 implies every t < 2^22 - 1/2: the magic
                    // rounding was exact; NaN fails the test too.
                    const bool big = __any_sync(tbk::kFull, !(acc < 4194303.0f));
                    const bool tie = __any_sync(tbk::kFull, dm == 0.5f);
                    const uint32_t sum_u =
                        __reduce_add_sync(tbk::kFull, magic_int(__fadd_rn(fminf(acc, 4194303.0f), kMagic)));
                    uint2 D = make_uint2(sum_u, sum_u);
                    uint32_t flags = 0;
                    if (b == tbk::kNoBinade) {
                        D = make_uint2(0u, 0u);
                        flags = kExact;
                    } else if (big) {
                        D = make_uint2(kSat, kSat);
                    } else if (tie) {
                        Fn fa{0u, 0u}, fb{0u, 0u};
#pragma unroll
                        for (int q = 0; q < 4; ++q) fa = compose(fa, term_fn(e[q], iu));
#pragma unroll
                        for (int q = 4; q < 8; ++q) fb = compose(fb, term_fn(e[q], iu));
                        fa = warp_compose(fa);
                        fb = warp_compose(fb);
                        const Fn ft = compose(fa, fb);
                        D = make_uint2(ft.a0, ft.a1);
                    }
                    if (lane == 0) {
                        R.D[t] = D;
                        if (flags) R.meta[t] = meta | flags;
                    }
                }
            }
            work_sync();
            // The summaries are complete: hand the row to its scanner.
            if (wt == 0) {
                __threadfence_block();
                tbk::mbar_arrive(&bar_ready[k]);
            }
        }
    }
}

// Shared memory besides the row buffer: summaries, tile sums, slots.
size_t staged_fixed(int nslot) {
    return kBufs * sizeof(RowSummary) + kMaxTiles * sizeof(float) +
           kBufs * (size_t)nslot * sizeof(Slot);
}

}  // namespace

namespace tbh {

// f32 softmax through k_softmax_staged.  Returns 1 (nothing launched) when
// the shape is not one it handles: a mask, more than 32768 columns, a
// column count that is not a multiple of 4, or unaligned rows.
int softmax_staged_f32(int64_t rows, int64_t cols, const float* x, float* y, cudaStream_t s) {
    if (cols > kMaxCols || cols % 4 || !aligned16(x) || !aligned16(y) || rows > INT32_MAX)
        return 1;
    DeviceState* ds = current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    const int ntiles = (int)((cols + kTileN - 1) / kTileN);
    const size_t xbytes = (size_t)ntiles * kTileN * 4;
    const size_t budget = ds->smem_optin > 1024 ? ds->smem_optin - 1024 : 0;  // static shared
    int nslot = ntiles < kMaxSlots ? ntiles : kMaxSlots;
    while (nslot > 2 && xbytes + staged_fixed(nslot) > budget) --nslot;
    if (nslot < 2 || xbytes + staged_fixed(nslot) > budget) return 1;
    const size_t smem = xbytes + staged_fixed(nslot);
    static thread_local size_t attr_set[64];
    if (ds->device >= 0 && ds->device < 64 && attr_set[ds->device] < smem) {
        TB_CUDA_TRY(cudaFuncSetAttribute(k_softmax_staged,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr_set[ds->device] = smem;
    }
    int per_sm = 0;
    TB_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_softmax_staged, kNT, smem));
    if (per_sm < 1) return 1;
    const int64_t cap = (int64_t)ds->sm_count * per_sm;
    const int grid = (int)(rows < cap ? rows : cap);
    k_softmax_staged<<<grid, kNT, smem, s>>>(x, y, (int)rows, (int)cols, nslot, ds->status);
    TB_LAUNCH_CHECK("softmax kernel (staged)");
    return TB_OK;
}

}  // namespace tbh
