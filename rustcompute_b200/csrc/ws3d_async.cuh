// ws3d_async.cuh -- cp.async-pipelined step kernel (one GPU or z-slabs).
//
// Same cell rule, arithmetic, shared-memory tile layout and chunk-major
// lockstep schedule as k_step_tma, but the stages are filled by every thread
// with 16-byte cp.async.cg copies (zero-filled outside the grid) instead of
// TMA, so the kernel also serves z-slabs, where this build keeps TMA out of
// multi-GPU code.  A ring of kAsyncStages stages runs kAsyncLook items ahead
// of the plane being computed, with one CTA barrier per plane.
//
// z-slabs: the (chunk, tile) items of the boundary z-chunks come after all
// interior items; right before the first copy of a boundary run the CTA waits
// (bounded) for the neighbour's flag, so interior work overlaps the exchange.
// Ghost planes are read with .cg copies (L2, coherent with the neighbour's
// peer stores).  Boundary planes are stored into the neighbours' ghost planes
// and fenced at system scope, exactly like k_step_zstream.
#pragma once

#include "ws3d_kernels.cuh"

namespace ws3d {

constexpr int kAsyncStages = 5;
constexpr int kAsyncLook = kAsyncStages - 2;

template <bool kC2F>
struct AsyncLayout {
    static constexpr int kPFloats = kAsyncPRow * (kAsyncTY + 2);  // 1360
    static constexpr int kTFloats = 128 * kAsyncTY;               // 1024
    static constexpr int kStageFloats = kPFloats + kTFloats * (kC2F ? 2 : 1);
    static constexpr int smem_bytes() { return kAsyncStages * kStageFloats * 4; }
};

__device__ __forceinline__ void cp_async16(float* smem_dst, const float* gsrc, bool valid) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
    const int n = valid ? 16 : 0;  // 0 source bytes: the 16 bytes are zero-filled
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(gsrc), "r"(n)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Walks a CTA's stage-items: per run, item 0 holds the pressure plane zs,
// item i >= 1 the front plane zs+i plus p_prev / c2 of plane zs+i-1.
struct AsyncCursor {
    uint32_t next_item;
    bool have;
    uint32_t tile, zs, ze, i;
};

struct AsyncSched {
    uint32_t tiles_x, tiles, clen, nchunks, nitems, nz;
    bool halo;
};

__device__ __forceinline__ bool cursor_run(AsyncCursor& c, const AsyncSched& s) {
    if (c.next_item >= s.nitems) {
        c.have = false;
        return false;
    }
    const uint32_t chunk = async_chunk_of(c.next_item, s.tiles, s.nchunks, s.halo);
    c.tile = c.next_item % s.tiles;
    c.zs = chunk * s.clen;
    c.ze = min(s.nz, c.zs + s.clen);
    c.i = 0;
    c.have = true;
    c.next_item += gridDim.x;
    return true;
}

__device__ __forceinline__ void cursor_next(AsyncCursor& c, const AsyncSched& s) {
    if (!c.have) return;
    if (c.i < c.ze - c.zs) {
        ++c.i;
        return;
    }
    cursor_run(c, s);
}

template <bool kC2F>
__global__ void __launch_bounds__(32 * kAsyncTY, 3)
k_step_async(StepParams a, AsyncSched sc) {
    using L = AsyncLayout<kC2F>;
    constexpr int S = kAsyncStages, LOOK = kAsyncLook;
    extern __shared__ float4 smem4[];  // 16-byte aligned, as cp.async needs
    float* smem = reinterpret_cast<float*>(smem4);

    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
    if (blockIdx.x >= sc.nitems) return;  // uniform over the CTA, before any barrier
    const bool halo_wait = a.wait_lo != nullptr || a.wait_hi != nullptr;
    const int64_t P = (int64_t)a.plane;
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);

    AsyncCursor is{blockIdx.x, false, 0, 0, 0, 0};
    AsyncCursor cs{blockIdx.x, false, 0, 0, 0, 0};
    cursor_run(is, sc);
    cursor_run(cs, sc);

    // This thread's copy assignments for the issue cursor's current run (they
    // depend on the tile only; per item only the plane offset changes).
    AsyncChunk cp0{}, cp1{}, ct{};
    bool has1 = false;
    uint32_t table_tile = 0xffffffffu;
    auto load_table = [&]() {
        if (!is.have || is.tile == table_tile) return;
        const uint32_t x0 = (is.tile % sc.tiles_x) * 128u;
        const uint32_t y0 = (is.tile / sc.tiles_x) * kAsyncTY;
        cp0 = async_p_chunk(t, x0, y0, a.H, a.pitch);
        has1 = t + 32 * kAsyncTY < kAsyncPChunks;
        if (has1) cp1 = async_p_chunk(t + 32 * kAsyncTY, x0, y0, a.H, a.pitch);
        ct = async_t_chunk(t, x0, y0, a.H, a.pitch);
        table_tile = is.tile;
    };

    // Issue the copies of the issue cursor's stage-item into stage (j % S);
    // every thread calls this at the same point, and commits one group.
    auto issue = [&](uint64_t j) {
        if (is.have) {
            if (is.i == 0 && halo_wait &&
                ((a.wait_lo && is.zs == 0) || (a.wait_hi && is.ze == a.nz))) {
                if (t == 0) {
                    unsigned int bad = 0;
                    if (a.wait_lo && is.zs == 0 && !wait_flag_geq(a.wait_lo, a.wait_val, a.budget_ns))
                        bad |= 1u;
                    if (a.wait_hi && is.ze == a.nz && !wait_flag_geq(a.wait_hi, a.wait_val, a.budget_ns))
                        bad |= 2u;
                    if (bad) atomicOr(a.status, bad);
                }
                __syncthreads();
            }
            load_table();
            float* st = smem + (j % S) * L::kStageFloats;
            const int64_t zp = (int64_t)is.zs + is.i;  // pressure plane of this item
            const float* psrc = a.p + zs_plane(zp, P);
            cp_async16(st + cp0.soff, cp0.valid ? psrc + cp0.goff : a.p, cp0.valid);
            if (has1) cp_async16(st + cp1.soff, cp1.valid ? psrc + cp1.goff : a.p, cp1.valid);
            if (is.i > 0) {
                const int64_t zo = zs_plane(zp - 1, P) + ct.goff;
                cp_async16(st + L::kPFloats + ct.soff, ct.valid ? a.pp + zo : a.pp, ct.valid);
                if (kC2F)
                    cp_async16(st + L::kPFloats + L::kTFloats + ct.soff,
                               ct.valid ? a.c2f + zo : a.c2f, ct.valid);
            }
            cursor_next(is, sc);
        }
        cp_async_commit();
    };

    uint64_t jiss = 0, j = 0;
    for (int k = 0; k < LOOK; ++k) issue(jiss++);

    while (cs.have) {
        const uint32_t x0 = (cs.tile % sc.tiles_x) * 128u, y0 = (cs.tile / sc.tiles_x) * kAsyncTY;
        const uint32_t x = x0 + 4u * lane, y = y0 + w;
        const bool act = x < a.pitch && y < a.H;
        const int64_t row = (int64_t)y * a.pitch + x;
        const XYPre xy = make_xypre(x, y, a);
        // The issue cursor passed this run's first item (and its flag wait)
        // before we got here, so the ghost plane zs-1 may be read now.
        float4 pm = act ? ld4_plane(a.p + zs_plane((int64_t)cs.zs - 1, P) + row,
                                    (int64_t)cs.zs - 1, a.nz)
                        : z4;
        cp_async_wait<LOOK - 1>();
        __syncthreads();
        issue(jiss++);
        const float* Pz = smem + (j % S) * L::kStageFloats;
        float4 pc = *reinterpret_cast<const float4*>(Pz + (w + 1) * kAsyncPRow + 4 + 4 * lane);
        ++j;
        for (uint32_t z = cs.zs; z < cs.ze; ++z, ++j) {
            cp_async_wait<LOOK - 1>();
            __syncthreads();
            issue(jiss++);
            const float* st = smem + (j % S) * L::kStageFloats;
            const float* Pz1 = st;
            const float* tPP = st + L::kPFloats;
            const float* tC2 = st + L::kPFloats + L::kTFloats;
            const float4 pn =
                *reinterpret_cast<const float4*>(Pz1 + (w + 1) * kAsyncPRow + 4 + 4 * lane);
            const float4 Sv = *reinterpret_cast<const float4*>(Pz + w * kAsyncPRow + 4 + 4 * lane);
            const float4 Nv =
                *reinterpret_cast<const float4*>(Pz + (w + 2) * kAsyncPRow + 4 + 4 * lane);
            const float4 vpp = *reinterpret_cast<const float4*>(tPP + w * 128 + 4 * lane);
            float4 vc2 = z4;
            if (kC2F) vc2 = *reinterpret_cast<const float4*>(tC2 + w * 128 + 4 * lane);
            float wl = __shfl_up_sync(0xffffffffu, pc.w, 1);
            float er = __shfl_down_sync(0xffffffffu, pc.x, 1);
            if (lane == 0) wl = Pz[(w + 1) * kAsyncPRow + 3];
            if (lane == 31) er = Pz[(w + 1) * kAsyncPRow + 4 + 128];
            if (act) {
                if (!kC2F) vc2 = make_float4(a.c2, a.c2, a.c2, a.c2);
                const float4 out = cells4_default(xy, a.z0 + z, wl, er, Sv, Nv, pm, pc, pn, vpp,
                                                  vc2, a);
                st4(a.pp + zs_plane((int64_t)z, P) + row, out);
                if (z == 0 && a.peer_lo) st4(a.peer_lo + row, out);
                if (z + 1 == a.nz && a.peer_hi) st4(a.peer_hi + row, out);
            }
            pm = pc;
            pc = pn;
            Pz = Pz1;
        }
        cursor_run(cs, sc);  // the consumer walks whole runs
    }
    cp_async_wait<0>();
    if (a.peer_lo || a.peer_hi) __threadfence_system();
}

}  // namespace ws3d
