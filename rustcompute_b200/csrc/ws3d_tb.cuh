// ws3d_tb.cuh -- two FDTD steps per launch (temporal blocking, depth 2), one
// GPU or a z-slab.
//
// Inputs A = p_t (pressure), B = p_{t-1} (pressure_prev) and c2; outputs
// X = p_{t+1} and Y = p_{t+2} go to two buffers that no CTA reads during the
// launch (neighbouring tiles still read A and B), so the context rotates over
// four field buffers.  HBM traffic per cell for two steps: read A, B, c2 once,
// write X and Y -- 20 bytes instead of 2 x 16.
//
// A CTA takes (z-chunk, tile) items in chunk-major order like k_step_tma; a
// tile is 128 x TY cells.  For a run of planes [zs, ze) the producer stages
// item i = 0 .. (ze - zs) + 3 as
//   A plane zs-2+i, a 136 x (TY+4) box from (x0-4, y0-2), and for i >= 2
//   B and c2 of plane q = zs-3+i, 136 x (TY+2) boxes from (x0-4, y0-1).
// Consumer warp w (0 .. TY+1) owns the extended row y0-1+w.  At item i >= 2 it
// computes X(q) on its row over the 128 core columns (a float4 per lane),
// keeping A(q-1), A(q) of its row in registers and reading A(q+1), the y
// neighbours, B and c2 from the stage.  The two halo-row warps (0 and TY+1)
// also compute the halo columns x0-1 and x0+128 of all TY+2 rows (ten lanes
// each, one cell per lane) into a small shared array.  Warps 1 .. TY then
// compute Y(q-1) on their (core) row: z neighbours X(q-2), X(q-1), X(q) from
// registers, y neighbours from a three-slot shared ring of X planes, x halo
// from the shared halo array, p_prev = A(q-1) from registers.  The ring is
// ordered by one mbarrier per slot instead of a CTA barrier per item: a warp
// stores X(q) into slot u % 3 (u counts its items), waits until every
// consumer warp has arrived on the slot of item u-1 (they stored X(q-1) and
// finished reading slot (u-2) % 3), computes Y(q-1) and arrives on slot u % 3.
// The slot a warp writes in item u was last read in item u-2, whose end it
// waited for in item u-1, so three slots need no second wait.  Warps drift up
// to about half an item apart, and with a fifth TMA stage that took 512^3 from
// 515 to 495 us per launch (neither change alone did: 4 stages with the split
// ring 518 us, 5 stages with a CTA barrier per item 514 us).  Cells use the
// lean rule of
// ws3d_lean.cuh (packed f32x2, same bits as the one-step kernels): the sponge
// factor is applied to every cell (1.0 outside it), lanes with boundary
// cells take a fix-up branch.  The item loop is
// unrolled three times so that the z queues rotate by renaming registers
// instead of moving them.
//
// Sources of step t are added to A and B by the host before the launch, like
// every step.  Sources of step t+1 are applied inside: X(src) += a in source
// order (also to the halo copies of X), and Y's p_prev A(src) += a/2 --
// exactly what injecting between the two steps does.  So one launch equals
// two steps bit for bit.  At most 32 sources (a shared table; lane k reads
// source k in tiles that hold one); the host checks.
//
// z-slabs (temporal depth 2, two ghost planes per side in every field
// buffer): X is also computed on ghost planes -1 / nz, from the two ghost
// planes of A on that side (stored there by the neighbour's previous launch)
// and the neighbour's own B and c2 planes, which the producer stages by TMA
// straight from the neighbour's buffers over NVLink (tensor maps over the
// mapped peer buffers; plain loads, no multicast -- B changes between
// launches and only its owner updates it, so no copy of it is kept here).  Y
// of planes 0, 1 / nz-2, nz-1 is also stored into the neighbour's Y buffer,
// i.e. its two ghost planes of the next launch's A.  Runs that read ghost
// planes or the neighbour's planes, or store into a neighbour, wait (bounded)
// for its flag, raised before its launch; those runs take a separate
// instance of the item code, interior runs the one-GPU code.  Equal to single
// steps bit for bit.
//
// Every wait is a bounded mbarrier wait; the item loop has no hardware
// barrier.  A consumer warp whose wait gives up stops arriving and leaves, so
// the other warps' waits on its arrivals give up too (warp 0 reports it), and
// so do the producer's waits for free stages.  The producer waits (bounded) for the copies it issued before it exits.  TMA
// loads never use multicast; they read this GPU's memory, and on z-slabs the
// neighbour's own edge planes of B and c2; default face layout.
#pragma once

#include "ws3d_lean.cuh"
#include "ws3d_tma.cuh"

namespace ws3d {

// Pipeline depth kS (stages of the TMA ring) is a template parameter; the
// host picks kTbStagesLo or kTbStagesHi from the size of the grid
// (tb_stages in ws3d_api.cu): a fifth stage in flight helps grids of up to
// about a gigabyte a field and costs time on larger ones.
#ifndef WS3D_TB_STAGES_HI
#define WS3D_TB_STAGES_HI 5
#endif
constexpr int kTbStagesLo = 4;
constexpr int kTbStagesHi = WS3D_TB_STAGES_HI;
constexpr int kTbXSlots = 3;      // slots of the shared X ring
constexpr int kTbRow = 136;       // floats per staged row (x0-4 .. x0+131)
constexpr int kTbMaxSrc = 32;     // sources per launch (one per lane)
constexpr int kTbSpongeMax = 64;  // sponge widths the kernel takes (table in shared memory)

template <bool kC2F, int kS>
struct TbLayout {
    static constexpr int kABytes = kTbRow * (kTbTY + 4) * 4;             // 6528
    static constexpr int kBBytes = kTbRow * (kTbTY + 2) * 4;             // 5440
    static constexpr int kBBytesPad = (kBBytes + 127) / 128 * 128;       // 5504
    static constexpr int kStage = kABytes + kBBytesPad * (kC2F ? 2 : 1);
    static constexpr int kTx = kABytes + kBBytes * (kC2F ? 2 : 1);
    static constexpr int kRingPlane = 128 * (kTbTY + 2);                 // floats
    static constexpr int kRingBytes = kTbXSlots * kRingPlane * 4;
    static constexpr int kHaloBytes = (kTbXSlots * (kTbTY + 2) * 2 * 4 + 127) / 128 * 128;  // [slot][TY+2][2]
    static constexpr int kTabBytes = kTbSpongeMax * 4;
    static constexpr int kSrcBytes = kTbMaxSrc * 16;
    // stages | X ring | X halo columns | sponge table | sources | 2*S + slots mbarriers | slack
    static constexpr int smem_bytes() {
        return kS * kStage + kRingBytes + kHaloBytes + kTabBytes + kSrcBytes + 16 * kS +
               8 * kTbXSlots + 128;
    }
};

struct TbArgs {
    StepParams a;             // p = A, pp = B (owned plane 0), c2f, geometry, sponge
    float* X;                 // owned plane 0 of the p_{t+1} output buffer
    float* Y;                 // owned plane 0 of the p_{t+2} output buffer
    const uint64_t* src_off;  // n_src slab offsets ((z+1)*plane + y*pitch + x), z in [-1, nz]
    const float* wavelet;     // n_src x wl_len
    uint32_t n_src;
    uint64_t wl_len;
    uint64_t step1;           // global index of step t+1
    uint32_t tiles_x, tiles, clen, nitems;
    int a_zoff;               // tensor-map z of A plane q is q + a_zoff
    // z-slabs (zero / null on one GPU).  X is also computed on the ghost
    // planes -1 / nz from the ghost planes of A and the neighbour's own B and
    // c2 planes (staged by TMA from its buffers: tmBlo / tmC2lo at plane
    // coordinate lo_nz, tmBhi / tmC2hi at 1); Y of the two first / last planes
    // is stored into the neighbour's Y buffer (its two ghost planes).
    uint32_t has_lo, has_hi;  // a lower / upper neighbour
    uint32_t lo_nz;           // the lower neighbour's owned planes
    float* peer_lo_y;         // lower neighbour's Y buffer at its first upper ghost plane
    float* peer_hi_y;         // upper neighbour's Y buffer at its first lower ghost plane
};


__device__ __forceinline__ float4 add_at(float4 v, int e, float d) {
    if (e == 0) v.x = __fadd_rn(v.x, d);
    else if (e == 1) v.y = __fadd_rn(v.y, d);
    else if (e == 2) v.z = __fadd_rn(v.z, d);
    else v.w = __fadd_rn(v.w, d);
    return v;
}

// kSlab: the z-slab instance (ghost-plane X, neighbour waits, pushes); the
// one-GPU instance compiles none of that into its item loop.
template <bool kC2F, bool kSlab, int kS>
__global__ void __launch_bounds__(32 * (kTbTY + 3), kTbCtasPerSm)
k_step_tma2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ CUtensorMap tmC2, const __grid_constant__ CUtensorMap tmBlo,
            const __grid_constant__ CUtensorMap tmBhi, const __grid_constant__ CUtensorMap tmC2lo,
            const __grid_constant__ CUtensorMap tmC2hi, TbArgs g) {
    using L = TbLayout<kC2F, kS>;
    constexpr int S = kS, TY = kTbTY, R = kTbRow;
    const StepParams& a = g.a;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~static_cast<uintptr_t>(127));
    float* ring = reinterpret_cast<float*>(smem + S * L::kStage);
    float* hring = reinterpret_cast<float*>(smem + S * L::kStage + L::kRingBytes);  // [2][TY+2][2]
    float* stab = reinterpret_cast<float*>(smem + S * L::kStage + L::kRingBytes + L::kHaloBytes);
    int4* srcs = reinterpret_cast<int4*>(smem + S * L::kStage + L::kRingBytes + L::kHaloBytes +
                                         L::kTabBytes);  // (x, y, local z, amplitude bits)
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * L::kStage + L::kRingBytes +
                                                 L::kHaloBytes + L::kTabBytes + L::kSrcBytes);
    uint64_t* empty = full + S;
    uint64_t* xbar = empty + S;  // X ring slot k: every consumer warp stored its X rows there

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (blockIdx.x >= g.nitems) return;  // uniform over the CTA, before any barrier
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], TY + 2);
        }
        for (int k = 0; k < kTbXSlots; ++k) mbar_init(&xbar[k], TY + 2);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < kTbSpongeMax)
        stab[threadIdx.x] = threadIdx.x < a.sponge_w ? a.sponge[threadIdx.x] : 1.0f;
    if (threadIdx.x < g.n_src) {
        // source k: slab offset ((z+1) * plane + y * pitch + x) -> coordinates
        const uint32_t k = threadIdx.x;
        const uint64_t off = g.src_off[k];
        const uint64_t pl = off / a.plane, rem = off - pl * a.plane;
        const uint32_t yy = (uint32_t)(rem / a.pitch);
        const float amp = g.step1 < g.wl_len ? g.wavelet[(uint64_t)k * g.wl_len + g.step1] : 0.0f;
        srcs[k] = make_int4((int)(rem - (uint64_t)yy * a.pitch), (int)yy, (int)pl - 1,
                            __float_as_int(amp));
    }
    __syncthreads();

    if (warp == TY + 2) {
        // ------------------------------------------------------------ producer
        if (lane != 0) return;
        uint32_t j = 0, s = 0, round = 0;  // items issued; stage and ring round of item j
        bool ok = true;
        for (uint32_t item = blockIdx.x; ok && item < g.nitems; item += gridDim.x) {
            // chunk-major on slabs too: measured on two B200s at 512^3 per GPU,
            // putting the boundary chunks last (as the one-step kernel does)
            // was 2.5 % slower -- the neighbours' flags are up by the time
            // the first chunk starts
            const uint32_t chunk = item / g.tiles, tile = item - chunk * g.tiles;
            const int zs = (int)(chunk * g.clen);
            const int ze = (int)min(a.nz, chunk * g.clen + g.clen);
            const int x0 = (int)((tile % g.tiles_x) * 128u), y0 = (int)((tile / g.tiles_x) * TY);
            // Runs that read ghost planes (A down to zs-2 / up to ze+1, the
            // neighbour's B and c2) or store into a neighbour's ghost planes
            // (Y of planes 0, 1 / nz-2, nz-1) wait for that neighbour's flag;
            // the acquire is then ordered before this thread's TMA loads of
            // our ghost planes and of the neighbour's planes.
            const bool need_lo = kSlab && a.wait_lo && zs < 2;
            const bool need_hi = kSlab && a.wait_hi && ze + 1 >= (int)a.nz;
            if (need_lo || need_hi) {
                unsigned int bad = 0;
                if (need_lo && !wait_flag_geq(a.wait_lo, a.wait_val, a.budget_ns, a.wait_acc)) bad |= 1u;
                if (need_hi && !wait_flag_geq(a.wait_hi, a.wait_val, a.budget_ns, a.wait_acc)) bad |= 2u;
                if (bad) atomicOr(a.status, bad);
                // the neighbour's stores into our ghost planes, acquired above,
                // before our TMA loads of them
                asm volatile("fence.proxy.async.global;" ::: "memory");
            }
            for (int i = 0; i <= ze - zs + 3; ++i) {
                if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1u)) {
                    ok = false;
                    break;
                }
                unsigned char* st = smem + s * L::kStage;
                const int zA = zs - 2 + i;  // A plane; tensor z = plane + a_zoff
                if (i < 2) {
                    mbar_expect_tx(&full[s], L::kABytes);
                    tma_load_3d(st, &tmA, x0 - 4, y0 - 2, zA + g.a_zoff, &full[s]);
                } else {
                    const int q = zA - 1;
                    mbar_expect_tx(&full[s], L::kTx);
                    tma_load_3d(st, &tmA, x0 - 4, y0 - 2, zA + g.a_zoff, &full[s]);
                    // B and c2 of plane q; of the ghost planes -1 / nz from the
                    // neighbour's own buffers (its last plane / its plane 0)
                    const CUtensorMap* mb = &tmB;
                    const CUtensorMap* mc = &tmC2;
                    int zb = q + 1;
                    if (kSlab && q < 0 && g.has_lo) {
                        mb = &tmBlo;
                        mc = &tmC2lo;
                        zb = (int)g.lo_nz;
                    } else if (kSlab && q >= (int)a.nz && g.has_hi) {
                        mb = &tmBhi;
                        mc = &tmC2hi;
                        zb = 1;
                    }
                    tma_load_3d(st + L::kABytes, mb, x0 - 4, y0 - 1, zb, &full[s]);
                    if (kC2F)
                        tma_load_3d(st + L::kABytes + L::kBBytesPad, mc, x0 - 4, y0 - 1, zb, &full[s]);
                }
                ++j;
                if (++s == S) {
                    s = 0;
                    ++round;
                }
            }
        }
        // A give-up leaves the consumers without items: their bounded waits end
        // the launch.  Do not leave while copies this thread issued may land.
        if (!ok) atomicOr(a.status, 4u);
        for (uint32_t q = j > (uint32_t)S ? j - S : 0u; q < j; ++q)
            mbar_wait(&full[q % S], (q / S) & 1u);
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int w = warp;  // extended row y0 - 1 + w
    const bool do_y = w >= 1 && w <= TY;
    const int64_t P = (int64_t)a.plane;
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    const f2 damp = pk(a.damping, a.damping);
    const int ecol = lane == 0 ? 3 : 132;  // x halo of lanes 0 / 31 (x0-1, x0+128)
    // halo-column cells: warps 0 and TY+1, lanes 0..TY+1, one (row, side) each
    const bool hwarp = w == 0 || w == TY + 1;
    const bool hlane = hwarp && lane < TY + 2;
    const int hrow = hlane ? (w == 0 ? 0 : (TY + 2) / 2) + (lane >> 1) : 0;
    const int hside = lane & 1;
    const int arow = (w + 1) * R;                        // this row in the A box
    const int hr = (hrow + 1) * R + (hside ? 132 : 3);  // the halo cell in the A box
    const bool has_src = (uint32_t)lane < g.n_src;       // lane k reads source k
    // plane sponge factor (planes 0 <= zg < Dg)
    auto fz_of = [&](uint32_t zg) -> float {
        const uint32_t dz = min(zg, a.Dg - 1 - zg);
        return dz < a.sponge_w ? stab[dz] : 1.0f;
    };

    // X planes this slab computes: its own, plus ghost plane -1 / nz next to a neighbour
    const int xlo = kSlab && g.has_lo ? -1 : 0;
    const int xhi = (int)a.nz + (kSlab && g.has_hi ? 1 : 0);
    uint32_t s = 0, ph = 0;  // stage and full-barrier parity of the current item
    uint32_t xs = 0, xph = 0;  // X ring slot of the current X item and its xbar parity
    bool xany = false;         // an earlier item stored X planes
    for (uint32_t item = blockIdx.x; item < g.nitems; item += gridDim.x) {
        const uint32_t chunk = item / g.tiles, tile = item - chunk * g.tiles;
        const int zs = (int)(chunk * g.clen);
        const int ze = (int)min(a.nz, chunk * g.clen + g.clen);
        const uint32_t x0 = (tile % g.tiles_x) * 128u, y0 = (tile / g.tiles_x) * TY;
        const uint32_t x = x0 + 4u * lane;
        const uint32_t y = y0 + (uint32_t)w - 1u;  // wraps for y0 = 0, w = 0: not a grid row
        const LeanRow lr = make_lean_row(x, y, a);
        const bool act = do_y && x < a.pitch && y < a.H;
        const int64_t row = (int64_t)y * a.pitch + x;  // + q * plane
        // halo cell of this lane (hlane only); x / y may wrap: not interior.
        // hf < 0 marks a halo cell that is not interior in x and y.
        float hf = -1.0f;
        {
            const uint32_t hx = hside ? x0 + 128u : x0 - 1u;
            const uint32_t hy = y0 + (uint32_t)hrow - 1u;
            if (lean_in(hx, a.W) && lean_in(hy, a.H))
                hf = sponge_f(min(min(hx, a.W - 1 - hx), min(hy, a.H - 1 - hy)), a);
        }
        // any source inside the tile's extended region (core + halo)?
        bool tile_src = false;
        if (g.n_src) {
            const int4 sc = has_src ? srcs[lane] : make_int4(-1000, -1000, 0, 0);
            tile_src = __any_sync(0xffffffffu, sc.x + 1 >= (int)x0 && sc.x <= (int)x0 + 128 &&
                                                   sc.y + 1 >= (int)y0 && sc.y <= (int)y0 + TY);
        }
        const int n = ze - zs;
        // this run stores Y planes into a neighbour's ghost planes
        const bool push_lo = kSlab && g.peer_lo_y != nullptr && zs < 2;
        const bool push_hi = kSlab && g.peer_hi_y != nullptr && ze + 2 > (int)a.nz;

        // Ends an item: release the previous item's stage (this warp no longer
        // reads it); after an X item, arrive on its ring slot (this warp's X
        // rows are stored and its reads of the previous slot are done); next
        // stage and slot.  True = a wait gave up: leave.
        auto end_item = [&](bool ok, bool release, bool xitem) -> bool {
            __syncwarp();
            if (lane == 0) {
                if (release) mbar_arrive(&empty[s == 0 ? S - 1 : s - 1]);
                if (xitem && ok) mbar_arrive(&xbar[xs]);
            }
            if (xitem) {
                xany = true;
                if (++xs == (uint32_t)kTbXSlots) {
                    xs = 0;
                    xph ^= 1u;
                }
            }
            if (++s == S) {
                s = 0;
                ph ^= 1u;
            }
            return !ok;
        };
        // Items 0, 1: A planes zs-2, zs-1 of this row (and of the halo cell).
        auto prologue = [&](float4& av, float& hv, bool release) -> bool {
            const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[s], ph));
            if (ok) {
                const float* Ac = reinterpret_cast<const float*>(smem + s * L::kStage);
                av = *reinterpret_cast<const float4*>(Ac + arow + 4 + 4 * lane);
                hv = hlane ? Ac[hr] : 0.f;
            }
            return end_item(ok, release, false);
        };
        // Item i >= 2: X(q), q = zs-3+i, from A(q-1) = a_m, A(q) = a_c and the
        // staged A(q+1) (kept in a_p); then Y(q-1) from X(q-2) = x_m,
        // X(q-1) = x_c and X(q) (kept in x_n).  Halo lanes: h_m, h_c, h_p.
        // tag (compile time): bit 0 kSrc, the tile holds a source, so the
        // sources of step t+1 are looked up (other tiles skip that code); bit
        // 1 kEdge, a slab run next to a neighbour (ghost-plane X, stores into
        // the neighbour) -- interior runs of a slab take the one-GPU code.
        auto body = [&](auto tag, int i, float4& a_m, float4& a_c, float4& a_p, float4& x_m,
                        float4& x_c, float4& x_n, float& h_m, float& h_c, float& h_p) -> bool {
            constexpr bool kSrc = (decltype(tag)::value & 1) != 0;
            constexpr bool kEdge = kSlab && (decltype(tag)::value & 2) != 0;
            bool ok = __all_sync(0xffffffffu, mbar_wait(&full[s], ph));
            if (ok) {
                const int q = zs - 3 + i;
                // X ring slots: this item's X(q) and the previous item's X(q-1)
                const uint32_t xw = xs;
                const uint32_t xr = xs == 0 ? kTbXSlots - 1 : xs - 1;
                const uint32_t sp = s == 0 ? S - 1 : s - 1;
                const float* Ac = reinterpret_cast<const float*>(smem + s * L::kStage);
                const float* Ap = reinterpret_cast<const float*>(smem + sp * L::kStage);
                const float* Bq = Ac + L::kABytes / 4;
                const float* Cq = Ac + (L::kABytes + L::kBBytesPad) / 4;
                a_p = *reinterpret_cast<const float4*>(Ac + arow + 4 + 4 * lane);
                h_p = hlane ? Ac[hr] : 0.f;
                x_n = z4;
                if (kEdge ? (q >= xlo && q < xhi) : (q >= 0 && q < (int)a.nz)) {
                    // ---- X(q) on extended row w
                    const uint32_t zg = a.z0 + (uint32_t)q;
                    const bool zin = zg >= 1 && zg + 1 < a.Dg;
                    const float fz = fz_of(zg);
                    const float4 sv = *reinterpret_cast<const float4*>(Ap + arow - R + 4 + 4 * lane);
                    const float4 nv = *reinterpret_cast<const float4*>(Ap + arow + R + 4 + 4 * lane);
                    const float4 bv = *reinterpret_cast<const float4*>(Bq + w * R + 4 + 4 * lane);
                    const float4 cq = kC2F ? *reinterpret_cast<const float4*>(Cq + w * R + 4 + 4 * lane)
                                           : make_float4(a.c2, a.c2, a.c2, a.c2);
                    const float ed = Ap[arow + ecol];
                    float wl = __shfl_up_sync(0xffffffffu, a_c.w, 1);
                    float er = __shfl_down_sync(0xffffffffu, a_c.x, 1);
                    if (lane == 0) wl = ed;
                    if (lane == 31) er = ed;
                    float4 xv = cells4_fast(wl, er, sv, nv, a_m, a_c, a_p, bv, cq, damp);
                    xv = cells4_finish(xv, lr.fx, fz, zin ? lr.bits : 0u, bv);
                    if (kSrc) {  // sources of step t+1: X += a, in source order
                        const int4 sc = has_src ? srcs[lane] : make_int4(0, -1, -1, 0);
                        unsigned mk = __ballot_sync(0xffffffffu, sc.z == q && sc.y == (int)y);
                        while (mk) {
                            const int k = __ffs(mk) - 1;
                            mk &= mk - 1;
                            const int dx = __shfl_sync(0xffffffffu, sc.x, k) - (int)x0;
                            const float amp = __int_as_float(__shfl_sync(0xffffffffu, sc.w, k));
                            if (dx >= 0 && dx < 128 && lane == (dx >> 2)) xv = add_at(xv, dx & 3, amp);
                        }
                    }
                    *reinterpret_cast<float4*>(ring + xw * L::kRingPlane + w * 128 + 4 * lane) = xv;
                    if (act && q >= zs && q < ze) st4(g.X + zs_plane(q, P) + row, xv);
                    x_n = xv;
                    if (hwarp) {
                        // ---- X(q) at the halo columns x0-1, x0+128 of rows 0 .. TY+1
                        float xh = 0.f;
                        if (hlane) {
                            const int br = hr - R;  // the halo cell in the B / c2 boxes
                            xh = cell1_lean(zin && hf >= 0.0f, fminf(hf, fz), Ap[hr - 1], Ap[hr + 1],
                                            Ap[hr - R], Ap[hr + R], h_m, h_p, h_c, Bq[br],
                                            kC2F ? Cq[br] : a.c2, a.damping);
                        }
                        if (kSrc) {
                            const int hx = (int)(hside ? x0 + 128u : x0 - 1u);
                            const int hy = (int)(y0 + (uint32_t)hrow - 1u);
                            const int4 sc = has_src ? srcs[lane] : make_int4(0, -1, -1, 0);
                            unsigned mk = __ballot_sync(0xffffffffu, sc.z == q);
                            while (mk) {
                                const int k = __ffs(mk) - 1;
                                mk &= mk - 1;
                                const int kx = __shfl_sync(0xffffffffu, sc.x, k);
                                const int ky = __shfl_sync(0xffffffffu, sc.y, k);
                                const float amp = __int_as_float(__shfl_sync(0xffffffffu, sc.w, k));
                                if (hlane && kx == hx && ky == hy) xh = __fadd_rn(xh, amp);
                            }
                        }
                        if (hlane) hring[(xw * (TY + 2) + hrow) * 2 + hside] = xh;
                    }
                }
                // every consumer warp stored its rows of X(q-1) and finished
                // reading the slot that X(q+1) will overwrite next item
                if (xany)
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait(&xbar[xr], xs == 0 ? xph ^ 1u : xph));
                // ---- Y(q-1) on core row w (shared X(q-1) written last item)
                const int qy = q - 1;
                if (ok && do_y && qy >= zs && qy < ze) {
                    const float* Xr = ring + xr * L::kRingPlane;
                    const float4 sv = *reinterpret_cast<const float4*>(Xr + (w - 1) * 128 + 4 * lane);
                    const float4 nv = *reinterpret_cast<const float4*>(Xr + (w + 1) * 128 + 4 * lane);
                    const float* Cp = reinterpret_cast<const float*>(smem + sp * L::kStage) +
                                      (L::kABytes + L::kBBytesPad) / 4;
                    const float4 c2y = kC2F ? *reinterpret_cast<const float4*>(Cp + w * R + 4 + 4 * lane)
                                            : make_float4(a.c2, a.c2, a.c2, a.c2);
                    const float eh = hring[(xr * (TY + 2) + w) * 2 + (lane == 31 ? 1 : 0)];
                    float wl = __shfl_up_sync(0xffffffffu, x_c.w, 1);
                    float er = __shfl_down_sync(0xffffffffu, x_c.x, 1);
                    if (lane == 0) wl = eh;
                    if (lane == 31) er = eh;
                    float4 pv = a_m;  // A(q-1)
                    if (kSrc) {  // sources of step t+1: p_prev += a/2
                        const int4 sc = has_src ? srcs[lane] : make_int4(0, -1, -1, 0);
                        unsigned mk = __ballot_sync(0xffffffffu, sc.z == qy && sc.y == (int)y);
                        while (mk) {
                            const int k = __ffs(mk) - 1;
                            mk &= mk - 1;
                            const int dx = __shfl_sync(0xffffffffu, sc.x, k) - (int)x0;
                            const float amp = __int_as_float(__shfl_sync(0xffffffffu, sc.w, k));
                            if (dx >= 0 && dx < 128 && lane == (dx >> 2))
                                pv = add_at(pv, dx & 3, __fmul_rn(amp, 0.5f));
                        }
                    }
                    const uint32_t zgy = a.z0 + (uint32_t)qy;
                    const float fzy = fz_of(zgy);
                    float4 yv = cells4_fast(wl, er, sv, nv, x_m, x_c, x_n, pv, c2y, damp);
                    yv = cells4_finish(yv, lr.fx, fzy, (zgy >= 1 && zgy + 1 < a.Dg) ? lr.bits : 0u,
                                       pv);
                    if (act) {
                        st4(g.Y + zs_plane(qy, P) + row, yv);
                        // the neighbours' two ghost planes of p_{t+2}
                        if (kEdge && push_lo && qy < 2)
                            st4(g.peer_lo_y + (int64_t)qy * P + row, yv);
                        if (kEdge && push_hi && qy + 2 >= (int)a.nz)
                            st4(g.peer_hi_y + ((int64_t)qy - (int64_t)a.nz + 1) * P + row, yv);
                    }
                }
            }
            return end_item(ok, true, true);
        };

        const int last = n + 3;

        float4 am = z4, ac = z4, ap = z4, xm = z4, xc = z4, xn = z4;
        float hm = 0.f, hc = 0.f, hp = 0.f;
        // Items 2 .. last, three per iteration (the z queues rotate by
        // renaming).
        auto run_items = [&](auto tag) -> bool {
            bool ab = false;
            int i = 2;
            for (; !ab && i + 2 <= last; i += 3) {
                ab = body(tag, i, am, ac, ap, xm, xc, xn, hm, hc, hp) ||
                     body(tag, i + 1, ac, ap, am, xc, xn, xm, hc, hp, hm) ||
                     body(tag, i + 2, ap, am, ac, xn, xm, xc, hp, hm, hc);
            }
            if (!ab && i <= last) ab = body(tag, i++, am, ac, ap, xm, xc, xn, hm, hc, hp);
            if (!ab && i <= last) ab = body(tag, i++, ac, ap, am, xc, xn, xm, hc, hp, hm);
            return ab;
        };
        bool abort = prologue(am, hm, false) || prologue(ac, hc, true);
        if (!abort) {
            using I0 = std::integral_constant<int, 0>;
            using I1 = std::integral_constant<int, 1>;
            if constexpr (kSlab) {
                using I2 = std::integral_constant<int, 2>;
                using I3 = std::integral_constant<int, 3>;
                if (zs < 2 || ze + 2 > (int)a.nz)
                    abort = tile_src ? run_items(I3{}) : run_items(I2{});
                else
                    abort = tile_src ? run_items(I1{}) : run_items(I0{});
            } else {
                abort = tile_src ? run_items(I1{}) : run_items(I0{});
            }
        }
        if (abort) {
            // a wait gave up; the other warps' waits on this warp's arrivals
            // give up in turn, so warp 0 reports it
            if (threadIdx.x == 0) atomicOr(a.status, 4u);
            return;
        }
        // the run's last stage
        if (lane == 0) mbar_arrive(&empty[s == 0 ? S - 1 : s - 1]);
    }
    // Warp 0 also waits for every warp's arrival on the CTA's last item, so a
    // warp that gave up there is reported as well.
    if (warp == 0 && xany &&
        !__all_sync(0xffffffffu, mbar_wait(&xbar[xs == 0 ? kTbXSlots - 1 : xs - 1],
                                           xs == 0 ? xph ^ 1u : xph)) &&
        lane == 0)
        atomicOr(a.status, 4u);
    if (kSlab && (g.peer_lo_y || g.peer_hi_y)) __threadfence_system();
}

}  // namespace ws3d
