// ws3d_async.cuh -- cp.async-pipelined step kernel (one GPU or z-slabs).
//
// Same cell rule, arithmetic, shared-memory tile layout and chunk-major
// lockstep schedule as k_step_tma, but the stages are filled by every thread
// with 16-byte cp.async.cg copies (zero-filled outside the grid) issued by a
// producer warp instead of TMA, so the kernel also serves z-slabs, where this
// build keeps TMA out of multi-GPU code.  Producer and consumer warps hand
// stages over through full/empty mbarriers, as in k_step_tma.
//
// z-slabs: the (chunk, tile) items of the boundary z-chunks come after all
// interior items; right before the first copy of a boundary run the CTA waits
// (bounded) for the neighbour's flag, so interior work overlaps the exchange.
// Ghost planes are read with .cg copies (L2, coherent with the neighbour's
// peer stores).  Boundary planes are stored into the neighbours' ghost planes
// and fenced at system scope, exactly like k_step_zstream.
#pragma once

#include "ws3d_kernels.cuh"
#include "ws3d_tma.cuh"  // mbarrier helpers

namespace ws3d {

constexpr int kAsyncStages = 4;

template <bool kC2F>
struct AsyncLayout {
    static constexpr int kPFloats = kAsyncPRow * (kAsyncTY + 2);  // 1360
    static constexpr int kTFloats = 128 * kAsyncTY;               // 1024
    static constexpr int kStageFloats = kPFloats + kTFloats * (kC2F ? 2 : 1);
    // stages, 2 * stages mbarriers, abort flag
    static constexpr int smem_bytes() { return kAsyncStages * kStageFloats * 4 + 16 * kAsyncStages + 16; }
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

__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// Producer-warp cp.async pipeline.  Warp TY (the producer) copies every
// stage with 32 lanes x 16-byte cp.async.cg (P: 340 chunks, p_prev / c2: 256
// chunks each, zero-filled outside the grid) and signals completion on the
// stage's full mbarrier with cp.async.mbarrier.arrive.noinc (count 32); the
// TY consumer warps are those of k_step_tma.  Waits are bounded.
template <bool kC2F>
__global__ void __launch_bounds__(32 * (kAsyncTY + 1), 3)
k_step_async(StepParams a, AsyncSched sc) {
    using L = AsyncLayout<kC2F>;
    constexpr int S = kAsyncStages;
    constexpr int TY = kAsyncTY;
    extern __shared__ float4 smem4[];  // 16-byte aligned, as cp.async needs
    float* smem = reinterpret_cast<float*>(smem4);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * L::kStageFloats);
    uint64_t* empty = full + S;
    int& abort_flag = *reinterpret_cast<int*>(empty + S);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (blockIdx.x >= sc.nitems) return;  // uniform over the CTA, before any barrier
    const int64_t P = (int64_t)a.plane;
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (threadIdx.x == 0) {
        for (int st = 0; st < S; ++st) {
            mbar_init(&full[st], 32);
            mbar_init(&empty[st], TY);
        }
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == TY) {
        // ------------------------------------------------------------ producer
        const bool halo_wait = a.wait_lo != nullptr || a.wait_hi != nullptr;
        AsyncCursor is{blockIdx.x, false, 0, 0, 0, 0};
        cursor_run(is, sc);
        uint64_t j = 0;
        bool ok = true;
        while (ok && is.have) {
            const uint32_t x0 = (is.tile % sc.tiles_x) * 128u;
            const uint32_t y0 = (is.tile / sc.tiles_x) * TY;
            if (is.i == 0 && halo_wait &&
                ((a.wait_lo && is.zs == 0) || (a.wait_hi && is.ze == a.nz))) {
                if (lane == 0) {
                    unsigned int bad = 0;
                    if (a.wait_lo && is.zs == 0 && !wait_flag_geq(a.wait_lo, a.wait_val, a.budget_ns, a.wait_acc))
                        bad |= 1u;
                    if (a.wait_hi && is.ze == a.nz && !wait_flag_geq(a.wait_hi, a.wait_val, a.budget_ns, a.wait_acc))
                        bad |= 2u;
                    if (bad) atomicOr(a.status, bad);
                }
                __syncwarp();
            }
            const int s = (int)(j % S);
            if (j >= S && !mbar_wait(&empty[s], (uint32_t)((j / S - 1) & 1))) {
                ok = false;
                break;
            }
            float* st = smem + s * L::kStageFloats;
            const int64_t zp = (int64_t)is.zs + is.i;
            const float* psrc = a.p + zs_plane(zp, P);
            for (int c = lane; c < kAsyncPChunks; c += 32) {
                const AsyncChunk ch = async_p_chunk(c, x0, y0, a.H, a.pitch);
                cp_async16(st + ch.soff, ch.valid ? psrc + ch.goff : a.p, ch.valid);
            }
            if (is.i > 0) {
                const int64_t zo = zs_plane(zp - 1, P);
                for (int c = lane; c < 32 * TY; c += 32) {
                    const AsyncChunk ch = async_t_chunk(c, x0, y0, a.H, a.pitch);
                    cp_async16(st + L::kPFloats + ch.soff, ch.valid ? a.pp + zo + ch.goff : a.pp,
                               ch.valid);
                    if (kC2F)
                        cp_async16(st + L::kPFloats + L::kTFloats + ch.soff,
                                   ch.valid ? a.c2f + zo + ch.goff : a.c2f, ch.valid);
                }
            }
            cp_async_mbar_arrive_noinc(&full[s]);
            ++j;
            cursor_next(is, sc);
        }
        if (!ok && lane == 0) {
            atomicOr(a.status, 4u);
            atomicExch(&abort_flag, 1);
        }
        // Leave only when this lane's copies have landed.
        cp_async_wait<0>();
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int w = warp;
    AsyncCursor cs{blockIdx.x, false, 0, 0, 0, 0};
    cursor_run(cs, sc);
    uint64_t j = 0;
    while (cs.have) {
        const uint32_t x0 = (cs.tile % sc.tiles_x) * 128u, y0 = (cs.tile / sc.tiles_x) * TY;
        const uint32_t x = x0 + 4u * lane, y = y0 + w;
        const bool act = x < a.pitch && y < a.H;
        const int64_t row = (int64_t)y * a.pitch + x;
        const XYPre xy = make_xypre(x, y, a);
        {
            const int s = (int)(j % S);
            if (!mbar_wait(&full[s], (uint32_t)((j / S) & 1)) || abort_flag) {
                atomicOr(a.status, 4u);
                return;
            }
        }
        // The producer passed this run's neighbour wait before its first copy,
        // so the ghost plane zs-1 may be read now.
        float4 pm = act ? ld4_plane(a.p + zs_plane((int64_t)cs.zs - 1, P) + row,
                                    (int64_t)cs.zs - 1, a.nz)
                        : z4;
        const float* Pz = smem + (j % S) * L::kStageFloats;
        float4 pc = *reinterpret_cast<const float4*>(Pz + (w + 1) * kAsyncPRow + 4 + 4 * lane);
        ++j;
        for (uint32_t z = cs.zs; z < cs.ze; ++z, ++j) {
            const int s = (int)(j % S);
            if (!mbar_wait(&full[s], (uint32_t)((j / S) & 1)) || abort_flag) {
                atomicOr(a.status, 4u);
                return;
            }
            const float* st = smem + s * L::kStageFloats;
            const float* Pz1 = st;
            const float* tPP = st + L::kPFloats;
            const float* tC2 = st + L::kPFloats + L::kTFloats;
            const float4 pn =
                *reinterpret_cast<const float4*>(Pz1 + (w + 1) * kAsyncPRow + 4 + 4 * lane);
            const float4 Sv = *reinterpret_cast<const float4*>(Pz + w * kAsyncPRow + 4 + 4 * lane);
            const float4 Nv =
                *reinterpret_cast<const float4*>(Pz + (w + 2) * kAsyncPRow + 4 + 4 * lane);
            const float4 vpp = *reinterpret_cast<const float4*>(tPP + w * 128 + 4 * lane);
            float4 vc2 = make_float4(a.c2, a.c2, a.c2, a.c2);
            if (kC2F) vc2 = *reinterpret_cast<const float4*>(tC2 + w * 128 + 4 * lane);
            float wl = __shfl_up_sync(0xffffffffu, pc.w, 1);
            float er = __shfl_down_sync(0xffffffffu, pc.x, 1);
            if (lane == 0) wl = Pz[(w + 1) * kAsyncPRow + 3];
            if (lane == 31) er = Pz[(w + 1) * kAsyncPRow + 4 + 128];
            if (act) {
                const float4 out = cells4_default(xy, a.z0 + z, wl, er, Sv, Nv, pm, pc, pn, vpp,
                                                  vc2, a);
                st4(a.pp + zs_plane((int64_t)z, P) + row, out);
                if (z == 0 && a.peer_lo) st4(a.peer_lo + row, out);
                if (z + 1 == a.nz && a.peer_hi) st4(a.peer_hi + row, out);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[(j - 1) % S]);
            pm = pc;
            pc = pn;
            Pz = Pz1;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[(j - 1) % S]);
        cursor_run(cs, sc);
    }
    if (a.peer_lo || a.peer_hi) __threadfence_system();
}

}  // namespace ws3d
