// ws3d_tma.cuh -- TMA-fed step kernel for one GPU or a z-slab (sm_100a).
//
// Same cell rule and arithmetic as k_step_zstream, different data movement:
//
//  * persistent grid over (z-chunk, tile) items in chunk-major order: tiles
//    that run together are neighbours in the same z-chunk and stream through
//    z in lockstep, so the halo rows a tile stages from its neighbours hit L2
//    (a tile-major balanced split re-read them from DRAM: +30 % traffic at
//    512^3); the chunk length is chosen so items divide evenly over the CTAs;
//  * one elected producer thread issues cp.async.bulk.tensor 3-D box loads
//    (no multicast, local memory only) into a ring of kStages shared-memory
//    stages: per plane the front pressure plane z+1 as a 136 x (TY+2) box
//    (x from x0-4 so the start stays 16-byte aligned, one halo row above and
//    below; out-of-range rows/columns arrive as zeros), and the 128 x TY
//    boxes of p_prev and c2 for plane z;
//  * TY consumer warps (one row each, a float4 per lane) keep the three-plane
//    register queue along z and read their y / x neighbours from the staged
//    plane; full/empty mbarriers hand stages between producer and consumers.
//
// Every mbarrier wait is bounded (try_wait with a suspend hint, iteration
// cap); a wait that gives up sets the status word, the CTA stops consuming,
// and the producer waits (bounded) for the copies it issued before exiting.
//
// z-slabs: the (chunk, tile) items of the two boundary z-chunks come after
// all interior items.  Before the first copy of a boundary run the producer
// waits (bounded) for the neighbour's flag, then fences the async proxy so
// that the TMA load of the upper ghost plane sees the neighbour's peer
// stores; consumers read the lower ghost plane through L2 after the run's
// first stage arrived (ordered after that wait).  Boundary planes are stored
// into the neighbours' ghost planes and fenced at system scope, like the
// other slab kernels; at temporal depth 2 the first two and last two planes
// are (the neighbours' two-step launches read two ghost planes per side).  All TMA loads read this GPU's own memory (the ghost
// planes are local buffers the neighbours write into); none uses multicast.
#pragma once

#include <cuda.h>

#include "ws3d_kernels.cuh"
#include "ws3d_lean.cuh"

namespace ws3d {

template <int TY, bool kC2F>
struct TmaLayout {
    // dynamic shared memory: stages, 2*S mbarriers, abort flag, alignment slack
    static constexpr int smem_bytes(int stages);
    static constexpr int kPRow = 136;                        // floats per staged P row
    static constexpr int kPBytes = kPRow * (TY + 2) * 4;
    static constexpr int kPBytesPad = (kPBytes + 127) / 128 * 128;
    static constexpr int kTBytes = 128 * TY * 4;             // p_prev / c2 tile
    static constexpr int kStage = kPBytesPad + kTBytes * (kC2F ? 2 : 1);
    static constexpr int kTxFull = kPBytes + kTBytes * (kC2F ? 2 : 1);
};

template <int TY, bool kC2F>
constexpr int TmaLayout<TY, kC2F>::smem_bytes(int stages) {
    return stages * kStage + 2 * stages * 8 + 16 + 128;
}

constexpr int kTmaStages = 4;
constexpr uint32_t kMbarSpins = 1u << 22;  // x ~0.5 us suspend hint: bounded to about 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bounded wait for the phase with parity `parity` to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    for (uint32_t it = 0; it < kMbarSpins; ++it) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n"
            " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(parity), "r"(500u)
            : "memory");
        if (done) return true;
    }
    return false;
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// Work items: item = chunk * tiles + tile (chunk-major, tile x fastest),
// covering planes [chunk * clen, min(nz, (chunk + 1) * clen)) of the tile.
// CTA c takes items c, c + G, c + 2G, ...  Items that run at the same time are
// neighbouring tiles of the same z-chunk, so the tiles advance through z in
// lockstep and the halo rows one tile stages from its neighbours are still in
// L2 when it needs them.
struct TmaRun {
    uint32_t tile, zs, ze;  // planes [zs, ze) of tile `tile`
};
// halo: boundary chunks after the interior ones (async_chunk_of).
__device__ __forceinline__ bool next_run(uint32_t& item, uint32_t nitems, uint32_t tiles,
                                         uint32_t clen, uint32_t nz, bool halo, TmaRun& r) {
    if (item >= nitems) return false;
    const uint32_t nchunks = (nz + clen - 1) / clen;
    const uint32_t chunk = async_chunk_of(item, tiles, nchunks, halo);
    r.tile = item % tiles;
    r.zs = chunk * clen;
    r.ze = min(nz, r.zs + clen);
    item += gridDim.x;
    return true;
}

// kLean: the packed cell rule of ws3d_lean.cuh (same bits; the host picks it
// when the sponge table is monotone), else cells4_default.
template <bool kC2F, int TY, bool kLean>
__global__ void __launch_bounds__(32 * (TY + 1), 3)
k_step_tma(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmPP,
           const __grid_constant__ CUtensorMap tmC2, StepParams a, uint32_t tiles_x,
           uint32_t tiles, uint32_t clen, uint32_t nitems) {
    using L = TmaLayout<TY, kC2F>;
    constexpr int S = kTmaStages;
    // Dynamic shared memory only (no static __shared__), rounded up to 128 B:
    // TMA destinations must be 128-byte aligned.
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~static_cast<uintptr_t>(127));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * L::kStage);
    uint64_t* empty = full + S;
    int& abort_flag = *reinterpret_cast<int*>(empty + S);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (blockIdx.x >= nitems) return;  // uniform over the CTA, before any barrier

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], TY);
        }
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const bool halo = a.wait_lo != nullptr || a.wait_hi != nullptr || a.peer_lo != nullptr ||
                      a.peer_hi != nullptr;
    if (warp == TY) {
        // ------------------------------------------------------------ producer
        if (lane != 0) return;
        uint64_t j = 0;  // stage items issued
        uint32_t item = blockIdx.x;
        TmaRun r;
        bool ok = true;
        while (ok && next_run(item, nitems, tiles, clen, a.nz, halo, r)) {
            const int x0 = (int)((r.tile % tiles_x) * 128u), y0 = (int)((r.tile / tiles_x) * TY);
            // runs that read a ghost plane or store into a neighbour's (two
            // planes per side at temporal depth 2) wait for that neighbour
            const bool need_lo = a.wait_lo && r.zs < (a.peer_lo2 ? 2u : 1u);
            const bool need_hi = a.wait_hi && r.ze + (a.peer_hi2 ? 1u : 0u) >= a.nz;
            if (need_lo || need_hi) {
                unsigned int bad = 0;
                if (need_lo && !wait_flag_geq(a.wait_lo, a.wait_val, a.budget_ns, a.wait_acc)) bad |= 1u;
                if (need_hi && !wait_flag_geq(a.wait_hi, a.wait_val, a.budget_ns, a.wait_acc)) bad |= 2u;
                if (bad) atomicOr(a.status, bad);
                // the neighbour's ghost-plane stores, acquired above, before our TMA loads
                asm volatile("fence.proxy.async.global;" ::: "memory");
            }
            for (uint32_t i = 0; ok && i <= r.ze - r.zs; ++i, ++j) {
                const int s = (int)(j % S);
                if (j >= S && !mbar_wait(&empty[s], (uint32_t)((j / S - 1) & 1))) {
                    ok = false;
                    break;
                }
                unsigned char* st = smem + s * L::kStage;
                if (i == 0) {  // prologue item: pressure plane zs
                    mbar_expect_tx(&full[s], L::kPBytes);
                    tma_load_3d(st, &tmP, x0 - 4, y0 - 1, (int)r.zs + 1, &full[s]);
                } else {       // plane z = zs + i - 1: pressure z+1, p_prev z, c2 z
                    const int z = (int)r.zs + (int)i - 1;
                    mbar_expect_tx(&full[s], L::kTxFull);
                    tma_load_3d(st, &tmP, x0 - 4, y0 - 1, z + 2, &full[s]);
                    tma_load_3d(st + L::kPBytesPad, &tmPP, x0, y0, z + 1, &full[s]);
                    if (kC2F)
                        tma_load_3d(st + L::kPBytesPad + L::kTBytes, &tmC2, x0, y0, z + 1,
                                    &full[s]);
                }
            }
        }
        if (!ok) {
            atomicOr(a.status, 4u);
            atomicExch(&abort_flag, 1);
        }
        // Do not leave while copies this thread issued may still be landing.
        const uint64_t first = j > (uint64_t)S ? j - S : 0;
        for (uint64_t q = first; q < j; ++q) mbar_wait(&full[q % S], (uint32_t)((q / S) & 1));
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int w = warp;
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    const int64_t P = (int64_t)a.plane;
    uint64_t j = 0;  // stage items consumed
    uint32_t item = blockIdx.x;
    TmaRun r;
    while (next_run(item, nitems, tiles, clen, a.nz, halo, r)) {
        const uint32_t x0 = (r.tile % tiles_x) * 128u, y0 = (r.tile / tiles_x) * TY;
        const uint32_t x = x0 + 4u * lane, y = y0 + w;
        const bool act = x < a.pitch && y < a.H;
        const int64_t row = (int64_t)y * a.pitch + x;
        XYPre xy{};
        LeanRow lr{};
        if (kLean) lr = make_lean_row(x, y, a);
        else xy = make_xypre(x, y, a);
        const float* pmp = a.p + zs_plane((int64_t)r.zs - 1, P) + row;  // plane zs-1
        // one GPU: issue the load early; slabs: plane -1 is a ghost plane, read
        // (through L2) once the producer has waited for the neighbour
        float4 pm = act && !halo ? ld4(pmp) : z4;
        // prologue item
        {
            const int s = (int)(j % S);
            if (!mbar_wait(&full[s], (uint32_t)((j / S) & 1))) {
                atomicOr(a.status, 4u);
                return;
            }
        }
        if (act && halo) pm = ld4_plane(pmp, (int64_t)r.zs - 1, a.nz);
        const float* Pz = reinterpret_cast<const float*>(smem + (j % S) * L::kStage);
        float4 pc = *reinterpret_cast<const float4*>(Pz + (w + 1) * L::kPRow + 4 + 4 * lane);
        ++j;
        for (uint32_t z = r.zs; z < r.ze; ++z, ++j) {
            const int s = (int)(j % S);
            if (!mbar_wait(&full[s], (uint32_t)((j / S) & 1)) || abort_flag) {
                atomicOr(a.status, 4u);
                return;
            }
            const unsigned char* st = smem + s * L::kStage;
            const float* Pz1 = reinterpret_cast<const float*>(st);
            const float* tPP = reinterpret_cast<const float*>(st + L::kPBytesPad);
            const float* tC2 = reinterpret_cast<const float*>(st + L::kPBytesPad + L::kTBytes);
            const float4 pn =
                *reinterpret_cast<const float4*>(Pz1 + (w + 1) * L::kPRow + 4 + 4 * lane);
            const float4 Sv = *reinterpret_cast<const float4*>(Pz + w * L::kPRow + 4 + 4 * lane);
            const float4 Nv =
                *reinterpret_cast<const float4*>(Pz + (w + 2) * L::kPRow + 4 + 4 * lane);
            const float4 vpp = *reinterpret_cast<const float4*>(tPP + w * 128 + 4 * lane);
            float4 vc2 = z4;
            if (kC2F) vc2 = *reinterpret_cast<const float4*>(tC2 + w * 128 + 4 * lane);
            float wl = __shfl_up_sync(0xffffffffu, pc.w, 1);
            float er = __shfl_down_sync(0xffffffffu, pc.x, 1);
            if (lane == 0) wl = Pz[(w + 1) * L::kPRow + 3];
            if (lane == 31) er = Pz[(w + 1) * L::kPRow + 4 + 128];
            if (act) {
                if (!kC2F) vc2 = make_float4(a.c2, a.c2, a.c2, a.c2);
                float4 out;
                if (kLean) {
                    const uint32_t zg = a.z0 + z;
                    out = cells4_fast(wl, er, Sv, Nv, pm, pc, pn, vpp, vc2,
                                      pk(a.damping, a.damping));
                    out = cells4_finish(out, lr.fx, lean_fz(zg, a), lean_mask(lr.bits, zg, a), vpp);
                } else {
                    out = cells4_default(xy, a.z0 + z, wl, er, Sv, Nv, pm, pc, pn, vpp, vc2, a);
                }
                st4(a.pp + zs_plane((int64_t)z, P) + row, out);
                if (z == 0 && a.peer_lo) st4(a.peer_lo + row, out);
                if (z + 1 == a.nz && a.peer_hi) st4(a.peer_hi + row, out);
                if (z == 1 && a.peer_lo2) st4(a.peer_lo2 + row, out);
                if (z + 2 == a.nz && a.peer_hi2) st4(a.peer_hi2 + row, out);
            }
            // The previous stage (plane z: neighbours, and this row's centre) is done.
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[(j - 1) % S]);
            pm = pc;
            pc = pn;
            Pz = Pz1;
        }
        // The last item of the run (plane ze) is consumed too.
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[(j - 1) % S]);
    }
    if (a.peer_lo || a.peer_hi) __threadfence_system();
}

}  // namespace ws3d
