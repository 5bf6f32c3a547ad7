// ws3d_persistent.cuh -- many FDTD steps in one cooperative launch.
//
// Replaces the reference's persistent FDTD kernel (crates/ringkernel-cuda-
// codegen/src/persistent_fdtd.rs:713-978, launched by ringkernel-cuda
// persistent.rs:1559-1640): every CTA loops over the steps, computes its
// (z-chunk, tile) items of the step with the z-streaming cell body, and meets
// the others at a software grid barrier.  The launch is cooperative, so all
// CTAs are co-resident and the barrier cannot deadlock; it is still bounded
// (%globaltimer budget), sets bit 3 of the status word when it gives up, and
// every CTA then leaves at the next barrier check.  The reference needs four
// grid barriers per step (halo pack/unpack through a global halo buffer); here
// neighbouring tiles read each other's planes straight from L2, so one barrier
// per step suffices (two when point sources are injected).
//
// z-slabs: CTA 0's leader raises the neighbours' flags before each step
// exactly like the per-step path (k_halo_signal), and the boundary items
// wait for the neighbours' flags inside zs_tile, so persistent and per-step
// calls can be mixed on the same slabs.
#pragma once

#include "ws3d_kernels.cuh"

namespace ws3d {

struct PersistentArgs {
    StepParams a;                 // geometry and constants; pointers set per step
    float* buf[2];                // slab bases (ghost plane -1) of the two field buffers
    float* lo_base[2];            // lower neighbour's buffers, or null
    float* hi_base[2];            // upper neighbour's buffers, or null
    uint64_t lo_ghost_off;        // lower neighbour: base -> its upper ghost plane
    unsigned long long* lo_flag;  // lower neighbour's flag this slab raises
    unsigned long long* hi_flag;  // upper neighbour's flag this slab raises
    unsigned long long halo_base; // halo steps taken before this launch
    unsigned int* bar_count;      // grid barrier: arrivals
    unsigned int* bar_gen;        // grid barrier: generation
    const uint64_t* src_off;
    const float* wavelet;
    const long long* src_ghost;
    uint32_t n_src;
    uint64_t wl_len;
    uint64_t step0;               // global step of the first step of the launch
    uint64_t nsteps;
    uint32_t cur0;                // buffer index holding the pressure at the start
    uint32_t tiles_x, tiles, clen, nitems;
};

__device__ __forceinline__ unsigned int ld_acquire_gpu_u32(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu_u32(unsigned int* p, unsigned int v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded grid barrier over all CTAs of a cooperative launch.  Returns false
// on every thread of a CTA whose leader gave up (status bit 3 set).
__device__ __forceinline__ bool grid_barrier(unsigned int* count, unsigned int* gen,
                                             unsigned int nblocks, unsigned long long budget_ns,
                                             unsigned int* status, int* s_ok) {
    __syncthreads();
    if (threadIdx.x == 0 && threadIdx.y == 0) {
        int ok = 1;
        const unsigned int g = ld_acquire_gpu_u32(gen);
        __threadfence();
        if (atomicAdd(count, 1u) == nblocks - 1) {
            atomicExch(count, 0u);
            __threadfence();
            st_release_gpu_u32(gen, g + 1u);
        } else {
            bool done = false;
            const unsigned long long t0 = global_ns();
            for (unsigned int it = 0; it < (1u << 26); ++it) {
                if (ld_acquire_gpu_u32(gen) != g) {
                    done = true;
                    break;
                }
                __nanosleep(32);
                if ((it & 63u) == 63u && global_ns() - t0 > budget_ns) break;
            }
            if (!done) {
                atomicOr(status, 8u);
                ok = 0;
            }
        }
        if (ok && *reinterpret_cast<volatile unsigned int*>(status) != 0u) ok = 0;
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

template <bool kC2F, bool kCells, int TY>
__global__ void __launch_bounds__(32 * TY, 3) k_persistent(PersistentArgs q) {
    __shared__ int s_ok;
    const unsigned int nb = gridDim.x;
    const bool leader = blockIdx.x == 0 && threadIdx.x == 0 && threadIdx.y == 0;
    const bool halo = q.lo_base[0] != nullptr || q.hi_base[0] != nullptr;
    for (uint64_t s = 0; s < q.nsteps; ++s) {
        const int cur = (int)((q.cur0 + s) & 1u);
        StepParams a = q.a;
        a.p = q.buf[cur] + a.plane;
        a.pp = q.buf[cur ^ 1] + a.plane;
        a.peer_lo = q.lo_base[0] ? q.lo_base[cur ^ 1] + q.lo_ghost_off : nullptr;
        a.peer_hi = q.hi_base[0] ? q.hi_base[cur ^ 1] : nullptr;
        a.wait_val = q.halo_base + s + 1;
        if (leader) {
            if (q.n_src)
                inject_sources_dev(q.buf[cur], q.buf[cur ^ 1], q.src_off, q.wavelet, q.n_src,
                                   q.wl_len, q.step0 + s, q.src_ghost, q.lo_base[cur],
                                   q.hi_base[cur]);
            if (halo) {
                __threadfence_system();
                if (q.lo_flag) st_release_sys(q.lo_flag, q.halo_base + s + 1);
                if (q.hi_flag) st_release_sys(q.hi_flag, q.halo_base + s + 1);
            }
        }
        if (q.n_src && !grid_barrier(q.bar_count, q.bar_gen, nb, a.budget_ns, a.status, &s_ok))
            return;
        for (uint32_t item = blockIdx.x; item < q.nitems; item += nb) {
            const uint32_t chunk = item / q.tiles, tile = item - chunk * q.tiles;
            const uint32_t zs = chunk * q.clen, ze = min(a.nz, zs + q.clen);
            zs_tile<kC2F, kCells, TY>(a, tile % q.tiles_x, tile / q.tiles_x, zs, ze);
        }
        if (!grid_barrier(q.bar_count, q.bar_gen, nb, a.budget_ns, a.status, &s_ok)) return;
    }
}

}  // namespace ws3d
