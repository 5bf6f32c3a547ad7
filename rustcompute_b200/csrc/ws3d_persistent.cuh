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
    unsigned long long* bar;      // grid barrier: arrivals (zeroed by the host before the launch)
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

__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Bounded grid barrier over all CTAs of a cooperative launch.  Each CTA's
// leader adds one arrival to a 64-bit counter that only grows (the host
// zeroes it before the launch) with release semantics, which publishes the
// CTA's writes, and polls the same counter with acquire loads until the
// round is complete, i.e. until it reaches the next multiple of the CTA
// count -- one atomic per CTA and no reset, generation word or last-arriver
// release on the critical path.  Then the status word: any error recorded
// before some CTA arrived is seen by every CTA after the round.  Returns
// false on every thread of a CTA whose leader gave up (status bit 3 set) or
// found an error.
__device__ __forceinline__ bool grid_barrier(unsigned long long* count, unsigned int nblocks,
                                             unsigned long long budget_ns, unsigned int* status,
                                             int* s_ok) {
    __syncthreads();
    if (threadIdx.x == 0 && threadIdx.y == 0) {
        int ok = 1;
        unsigned long long old;
        asm volatile("atom.add.release.gpu.global.u64 %0, [%1], 1;"
                     : "=l"(old)
                     : "l"(count)
                     : "memory");
        const unsigned long long target = (old / nblocks + 1ull) * nblocks;
        if (ld_acquire_gpu_u64(count) < target) {
            bool done = false;
            const unsigned long long t0 = global_ns();
            for (unsigned int it = 0; it < (1u << 26); ++it) {
                __nanosleep(32);
                if (ld_acquire_gpu_u64(count) >= target) {
                    done = true;
                    break;
                }
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
                                   q.hi_base[0] ? q.hi_base[cur] - a.plane : nullptr);
            if (halo) {
                __threadfence_system();
                if (q.lo_flag) st_release_sys(q.lo_flag, q.halo_base + s + 1);
                if (q.hi_flag) st_release_sys(q.hi_flag, q.halo_base + s + 1);
            }
        }
        if (q.n_src && !grid_barrier(q.bar, nb, a.budget_ns, a.status, &s_ok))
            return;
        for (uint32_t item = blockIdx.x; item < q.nitems; item += nb) {
            const uint32_t chunk = item / q.tiles, tile = item - chunk * q.tiles;
            const uint32_t zs = chunk * q.clen, ze = min(a.nz, zs + q.clen);
            zs_tile<kC2F, kCells, TY>(a, tile % q.tiles_x, tile / q.tiles_x, zs, ze);
        }
        if (!grid_barrier(q.bar, nb, a.budget_ns, a.status, &s_ok)) return;
    }
}

// ---------------------------------------------------------------------------
// Block-parallel persistent step (default face layout).
//
// k_persistent's z-streaming items walk a run of planes through a register
// queue: on a small, L2-resident grid (config 5, 128^3) every step is then a
// chain of dependent plane loads per CTA.  Here a step is a flat set of
// blocks -- NW rows (one per warp) of 128 cells of one plane z at one x-tile --
// spread over the CTAs; each row issues all its loads at once (centre, z
// neighbours, p_prev, c2, the two x-halo cells), the y neighbours come from
// the other rows of the block through shared memory, so a step costs about
// one L2 round trip plus the grid barrier.  The cell rule is cells4_default,
// the same operations in the same order as every other kernel here.
//
// Fields are rewritten every step inside the launch, so they are read
// through L2 (ld.global.cg): no SM's L1 can hold a value from an earlier
// step.  On z-slabs the blocks of the first and last owned plane (they read
// the ghost planes a neighbour stores into, and store into the neighbour's
// ghost planes) run after the interior blocks of the step; a CTA waits
// (bounded) for the neighbour's flag once before its first such block.
// ---------------------------------------------------------------------------
constexpr int kRowThreads = 512;

__device__ __forceinline__ float4 ldcg4(const float* p) {
    return __ldcg(reinterpret_cast<const float4*>(p));
}

// One step over the blocks cta, cta + ncta, ... of the step's block list;
// warp w of the CTA computes row w of each block.  The block's rows of the
// current pressure are shared through shared memory, so each row loads its
// own p, its z neighbours, p_prev (and c2) from L2, and the y neighbours come
// from the rows the other warps loaded (plus two halo rows per block).
template <bool kC2F, int NW>
__device__ __forceinline__ void step_rows(const StepParams& a, uint32_t tiles_x, bool halo,
                                          uint32_t w, uint32_t cta, uint32_t ncta) {
    __shared__ float4 srow[NW + 2][32];
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t yblocks = (a.H + NW - 1) / NW;
    const uint64_t nblk = (uint64_t)yblocks * tiles_x * a.nz;
    const int64_t P = (int64_t)a.plane;
    const int64_t pitch = (int64_t)a.pitch;
    const float* __restrict__ p = a.p;
    float* __restrict__ pp = a.pp;
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    bool waited_lo = a.wait_lo == nullptr, waited_hi = a.wait_hi == nullptr;
    for (uint64_t blk = cta; blk < nblk; blk += ncta) {
        const RowCoord rc = row_coord(blk, yblocks, tiles_x, a.nz, halo);
        const uint32_t z = rc.z, y0 = rc.yb * NW, y = y0 + w;
        const uint32_t x0 = rc.tx * 128u, x = x0 + 4u * lane;
        if (halo) {  // CTA-uniform: one bounded wait per neighbour and step
            const bool lo = z == 0 && !waited_lo, hi = z + 1 == a.nz && !waited_hi;
            if (lo || hi) {
                if (threadIdx.x == 0 && threadIdx.y == 0) {
                    unsigned int bad = 0;
                    if (lo && !wait_flag_geq(a.wait_lo, a.wait_val, a.budget_ns, a.wait_acc))
                        bad |= 1u;
                    if (hi && !wait_flag_geq(a.wait_hi, a.wait_val, a.budget_ns, a.wait_acc))
                        bad |= 2u;
                    if (bad) atomicOr(a.status, bad);
                }
                __syncthreads();
                waited_lo = waited_lo || lo;
                waited_hi = waited_hi || hi;
            }
        }
        const bool xin = x < a.pitch;
        const bool act = xin && y < a.H;
        const int64_t o = (int64_t)z * P + (int64_t)y * pitch + x;
        float4 pc = z4, pm = z4, pn = z4, vpp = z4;
        float4 c2v = make_float4(a.c2, a.c2, a.c2, a.c2);
        float hl = 0.f, hr = 0.f;
        if (act) {
            pc = ldcg4(p + o);
            pm = ldcg4(p + o - P);
            pn = ldcg4(p + o + P);
            vpp = ldcg4(pp + o);
            if (kC2F) c2v = __ldg(reinterpret_cast<const float4*>(a.c2f + o));
            if (lane == 0 && x0 > 0) hl = __ldcg(p + o - 1);
            if (lane == 31 && x0 + 128u < a.pitch) hr = __ldcg(p + o + 4);
        }
        // halo rows y0 - 1 and y0 + NW: inside the allocation (the ghost planes
        // frame the owned ones); at the faces y = 0 / H - 1 they are not used
        float4 hy = z4;
        if (xin && w == 0) hy = ldcg4(p + (int64_t)z * P + ((int64_t)y0 - 1) * pitch + x);
        if (xin && w == NW - 1 && y0 + NW <= a.H)
            hy = ldcg4(p + (int64_t)z * P + ((int64_t)y0 + NW) * pitch + x);
        srow[w + 1][lane] = pc;
        if (w == 0) srow[0][lane] = hy;
        if (w == NW - 1) srow[NW + 1][lane] = hy;
        float wl = __shfl_up_sync(0xffffffffu, pc.w, 1);
        float er = __shfl_down_sync(0xffffffffu, pc.x, 1);
        if (lane == 0) wl = hl;
        if (lane == 31) er = hr;
        __syncthreads();
        if (act) {
            const float4 S = srow[w][lane], N = srow[w + 2][lane];
            const XYPre xy = make_xypre(x, y, a);
            const float4 out = cells4_default(xy, a.z0 + z, wl, er, S, N, pm, pc, pn, vpp, c2v, a);
            st4(pp + o, out);
            const int64_t ro = (int64_t)y * pitch + x;
            if (z == 0 && a.peer_lo) st4(a.peer_lo + ro, out);
            if (z + 1 == a.nz && a.peer_hi) st4(a.peer_hi + ro, out);
        }
        __syncthreads();  // the next block's rows overwrite srow
    }
}

template <bool kC2F>
__global__ void __launch_bounds__(kRowThreads, 2) k_persistent_rows(PersistentArgs q) {
    __shared__ int s_ok;
    const unsigned int nb = gridDim.x;
    const bool leader = blockIdx.x == 0 && threadIdx.x == 0;
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
                                   q.hi_base[0] ? q.hi_base[cur] - a.plane : nullptr);
            if (halo) {
                __threadfence_system();
                if (q.lo_flag) st_release_sys(q.lo_flag, q.halo_base + s + 1);
                if (q.hi_flag) st_release_sys(q.hi_flag, q.halo_base + s + 1);
            }
        }
        if (q.n_src && !grid_barrier(q.bar, nb, a.budget_ns, a.status, &s_ok))
            return;
        step_rows<kC2F, kRowThreads / 32>(a, q.tiles_x, halo, threadIdx.x >> 5, blockIdx.x, nb);
        if (!grid_barrier(q.bar, nb, a.budget_ns, a.status, &s_ok)) return;
    }
}

// ---------------------------------------------------------------------------
// Resident (command-driven) kernel.
//
// The reference keeps its persistent kernel running and feeds it commands
// through SPSC queues in mapped host memory (persistent_fdtd.rs:766-812,
// 917-978; host side ringkernel-cuda persistent.rs:571-1050).  k_resident
// does the same on one GPU: between steps the leader thread (CTA 0, thread 0)
// drains the H2K queue, decides "step", "idle" or "exit" and publishes the
// decision before the per-step grid barrier; the step itself is the
// row-parallel body of k_persistent_rows (default faces) or the z-streaming
// body of k_persistent (cell arrays), so fields are bit-identical to
// ws3d_step.  Every progress_interval steps all CTAs sum p^2 (fixed order,
// double) and the leader posts a PROGRESS message.  Waits are bounded: the
// grid barrier as in k_persistent, and an idle kernel (no steps, not paused
// for work) leaves after idle_budget_ns; the host relaunches it when work
// arrives.  Mapped memory is read with .sys-scope acquire / volatile loads
// and written with posted volatile stores plus a release of the queue index.
// ---------------------------------------------------------------------------
struct ResidentCtrl {            // 256 bytes, mapped host memory
    uint32_t should_terminate;
    uint32_t paused;
    uint64_t steps_remaining;
    uint64_t current_step;
    uint32_t current_buffer;     // pressure role relative to the launch (0 or 1)
    uint32_t has_terminated;     // the kernel has left (any reason)
    float total_energy;
    uint32_t exit_reason;        // 0 running, 1 TERMINATE, 2 idle budget, 3 barrier gave up
    uint64_t messages_processed;
    uint64_t k2h_dropped;
    uint64_t steps_run;          // steps run by this launch
    uint64_t reserved[24];
};
static_assert(sizeof(ResidentCtrl) == 256, "control block layout");

struct ResQueue {                // 128 bytes (SpscQueueHeader, persistent_fdtd.rs:224-231)
    uint64_t head;               // consumer index
    uint64_t tail;               // producer index
    uint32_t capacity;
    uint32_t mask;
    uint64_t pad[13];
};
static_assert(sizeof(ResQueue) == 128, "queue header layout");

struct ResMsg {                  // 64-byte H2K / K2H slot, read and written as 4 x 16 bytes
    uint4 q[4];
};

struct ResidentArgs {
    PersistentArgs q;            // one GPU: no neighbours
    ResidentCtrl* ctrl;
    ResQueue* h2k;
    const ResMsg* h2k_slots;
    ResQueue* k2h;
    ResMsg* k2h_slots;
    unsigned int* decision;      // device word written by the leader before each barrier
    double* partial;             // per-CTA energy partials (>= gridDim.x)
    uint64_t progress_interval;
    unsigned long long idle_budget_ns;
    uint32_t h2k_mask;           // queue capacities - 1 (kept off the PCIe path)
    uint32_t k2h_capacity;
};

// The leader thread's copy of the control state, in shared memory so that
// the other threads do not carry it in registers through the step.
constexpr uint32_t kResMaxPending = 64;  // impulses queued between two barriers
struct ResLeader {
    uint64_t steps_rem, msgs, dropped, h2k_head, k2h_tail, k2h_head;
    unsigned long long idle_t0;
    uint32_t paused, term, npend;
    float energy;
    uint4 pend[kResMaxPending];  // (x, y, z, amplitude bits)
};

enum : unsigned int { kResIdle = 0, kResStep = 1, kResExitTerm = 2, kResExitIdle = 3 };

// 16-byte volatile accesses to mapped host memory (queue slots)
__device__ __forceinline__ uint4 ld_volatile_v4(const void* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ void st_volatile_v4(void* p, uint4 v) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ uint64_t ld_acquire_sys_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Leader: post one K2H message (dropped, and counted, when the queue is full).
__device__ __forceinline__ void res_post(const ResidentArgs& r, uint64_t& tail, uint64_t& head_seen,
                                         uint64_t& dropped, uint32_t type, uint64_t cmd_id,
                                         uint64_t step, uint64_t remaining, float energy,
                                         uint32_t error) {
    const uint64_t cap = r.k2h_capacity;
    if (tail - head_seen >= cap) head_seen = ld_acquire_sys_u64(&r.k2h->head);
    if (tail - head_seen >= cap) {
        ++dropped;
        return;
    }
    ResMsg m;
    m.q[0] = make_uint4(type, 0u, (uint32_t)cmd_id, (uint32_t)(cmd_id >> 32));
    m.q[1] = make_uint4((uint32_t)step, (uint32_t)(step >> 32), (uint32_t)remaining,
                        (uint32_t)(remaining >> 32));
    m.q[2] = make_uint4(__float_as_uint(energy), error, 0u, 0u);
    m.q[3] = make_uint4(0u, 0u, 0u, 0u);
    uint4* dst = r.k2h_slots[tail & (cap - 1)].q;
    for (int k = 0; k < 4; ++k) st_volatile_v4(dst + k, m.q[k]);
    ++tail;
    st_release_sys_u64(&r.k2h->tail, tail);  // orders the slot stores before the index
}

// All CTAs: sum of p^2 over the owned cells of `p` (owned plane 0), fixed
// order; returns the total on the leader.  Two grid barriers.
template <int TY>
__device__ __forceinline__ bool res_energy(const ResidentArgs& r, const float* p, double* out,
                                           int* s_ok) {
    __shared__ double s_part[TY];
    const PersistentArgs& q = r.q;
    const StepParams& a = q.a;
    const unsigned int nb = gridDim.x;
    const int t = threadIdx.y * 32 + threadIdx.x;
    double acc = 0.0;
    const uint64_t rows = (uint64_t)a.nz * a.H;
    for (uint64_t row = blockIdx.x; row < rows; row += nb) {
        const uint64_t z = row / a.H, y = row - z * a.H;
        const float* pr = p + z * a.plane + y * a.pitch;
        for (uint32_t x = (uint32_t)t; x < a.W; x += 32u * TY) {
            const float v = pr[x];
            acc += (double)v * (double)v;
        }
    }
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
    if (threadIdx.x == 0) s_part[threadIdx.y] = acc;
    __syncthreads();
    if (t == 0) {
        double b = 0.0;
        for (int k = 0; k < TY; ++k) b += s_part[k];
        r.partial[blockIdx.x] = b;
    }
    if (!grid_barrier(q.bar, nb, a.budget_ns, a.status, s_ok)) return false;
    if (blockIdx.x == 0 && t == 0) {
        double e = 0.0;
        for (unsigned int k = 0; k < nb; ++k) e += r.partial[k];
        *out = e;
    }
    return true;
}

template <bool kC2F, bool kCells, int TY>
__global__ void __launch_bounds__(32 * TY, 3) k_resident(ResidentArgs r) {
    __shared__ int s_ok;
    __shared__ unsigned int s_op;
    __shared__ ResLeader L;  // used by the leader thread of CTA 0 only
    const PersistentArgs& q = r.q;
    const unsigned int nb = gridDim.x;
    const bool leader = blockIdx.x == 0 && threadIdx.x == 0 && threadIdx.y == 0;
    const uint64_t interval = r.progress_interval ? r.progress_interval : 100;

    // The leader's copy of the control state (mapped memory is read once here).
    volatile ResidentCtrl* ctrl = r.ctrl;
    if (leader) {
        L.steps_rem = ctrl->steps_remaining;
        L.paused = ctrl->paused;
        L.term = 0;
        L.npend = 0;
        L.msgs = ctrl->messages_processed;
        L.dropped = ctrl->k2h_dropped;
        L.energy = ctrl->total_energy;
        L.h2k_head = ld_acquire_sys_u64(&r.h2k->head);
        L.k2h_tail = ld_acquire_sys_u64(&r.k2h->tail);
        L.k2h_head = ld_acquire_sys_u64(&r.k2h->head);
        L.idle_t0 = global_ns();
    }
    int cur = 0;           // role of the pressure buffer (0 = q.buf[0] at launch)
    uint64_t ran = 0;      // steps run by this launch (same on every CTA)
    unsigned int op = kResIdle, pre = 0;
    uint64_t tail_hint = 0;  // leader: H2K tail read at the start of the step (relaxed)

    // Leader: drain the H2K commands up to `tail` and decide what the grid
    // does next (persistent_fdtd.rs:769-823).  Impulses are queued and applied
    // after the next grid barrier, when no CTA is computing.
    auto decide = [&](uint64_t tail) {
        if (tail != L.h2k_head) asm volatile("fence.acq_rel.sys;" ::: "memory");
        while (L.h2k_head != tail) {
            const uint4* src = r.h2k_slots[L.h2k_head & r.h2k_mask].q;
            const uint4 m0 = ld_volatile_v4(src), m1 = ld_volatile_v4(src + 1),
                        m2 = ld_volatile_v4(src + 2);
            const uint32_t cmd = m0.x;
            if (cmd == 5u && L.npend == kResMaxPending) break;  // full: leave it queued
            const uint64_t cmd_id = (uint64_t)m0.z | ((uint64_t)m0.w << 32);
            const uint64_t param1 = (uint64_t)m1.x | ((uint64_t)m1.y << 32);
            ++L.h2k_head;
            ++L.msgs;
            switch (cmd) {
                case 0: break;                                   // NOP
                case 1: L.steps_rem += param1; break;            // RUN_STEPS
                case 2: L.paused = 1; break;                     // PAUSE
                case 3: L.paused = 0; break;                     // RESUME
                case 4: L.term = 1; break;                       // TERMINATE
                case 5:                                          // INJECT_IMPULSE
                    L.pend[L.npend++] = make_uint4((uint32_t)(param1 >> 32), (uint32_t)param1, m1.z,
                                                   m2.x);
                    break;
                case 7:                                          // GET_PROGRESS
                    res_post(r, L.k2h_tail, L.k2h_head, L.dropped, 1u, cmd_id, q.step0 + ran,
                             L.steps_rem, L.energy, 0u);
                    break;
                default:                                         // SET_SOURCE, unknown
                    res_post(r, L.k2h_tail, L.k2h_head, L.dropped, 2u, cmd_id, q.step0 + ran,
                             L.steps_rem, L.energy, cmd);
                    break;
            }
        }
        st_release_sys_u64(&r.h2k->head, L.h2k_head);
        ctrl->paused = L.paused;
        ctrl->steps_remaining = L.steps_rem;
        ctrl->messages_processed = L.msgs;
        unsigned int next;
        if (L.term) {
            next = kResExitTerm;
        } else if (L.steps_rem > 0 && !L.paused) {
            next = kResStep;
            L.idle_t0 = global_ns();
        } else if (global_ns() - L.idle_t0 > r.idle_budget_ns && L.h2k_head == tail) {
            next = kResExitIdle;
        } else {
            next = kResIdle;
        }
        *reinterpret_cast<volatile unsigned int*>(r.decision) = next | (L.npend ? 0x100u : 0u);
    };
    // Leader: the queued impulses, in command order (ws3d_inject_impulse's
    // semantics: p += a, p_prev += a/2).
    auto apply_pending = [&]() {
        for (uint32_t k = 0; k < L.npend; ++k) {
            const uint4 e = L.pend[k];
            if (e.x < q.a.W && e.y < q.a.H && e.z < q.a.Dg) {
                const uint64_t off =
                    (uint64_t)(e.z + 1) * q.a.plane + (uint64_t)e.y * q.a.pitch + e.x;
                float* pc = q.buf[cur] + off;
                float* pp = q.buf[cur ^ 1] + off;
                const float amp = __uint_as_float(e.w);
                *pc = __fadd_rn(*pc, amp);
                *pp = __fadd_rn(*pp, __fmul_rn(amp, 0.5f));
            }
        }
        L.npend = 0;
    };
    // Barrier that also hands the leader's decision to every thread.
    auto barrier_decision = [&]() -> bool {
        if (!grid_barrier(q.bar, nb, q.a.budget_ns, q.a.status, &s_ok))
            return false;
        if (threadIdx.x == 0 && threadIdx.y == 0)
            s_op = *reinterpret_cast<volatile unsigned int*>(r.decision);
        __syncthreads();
        op = s_op & 0xFFu;
        pre = s_op >> 8;
        return true;
    };

    if (leader) decide(ld_acquire_sys_u64(&r.h2k->tail));
    bool ok = barrier_decision();
    while (ok) {
        if (pre && leader) apply_pending();
        if (op == kResExitTerm || op == kResExitIdle) {
            // the final energy reads the impulses just applied
            if (pre && !grid_barrier(q.bar, nb, q.a.budget_ns, q.a.status, &s_ok))
                ok = false;
            break;
        }
        if (op != kResStep) {  // idle: sleep, poll again
            if (leader) {
                __nanosleep(20000);
                decide(ld_acquire_sys_u64(&r.h2k->tail));
            }
            ok = barrier_decision();
            continue;
        }

        // ---- one step (k_persistent's body, one GPU); one grid barrier, plus
        // one when sources or queued impulses must land first
        if (leader)  // read ahead: the PCIe round trip overlaps the step
            tail_hint = *reinterpret_cast<volatile const uint64_t*>(&r.h2k->tail);
        StepParams a = q.a;
        a.p = q.buf[cur] + a.plane;
        a.pp = q.buf[cur ^ 1] + a.plane;
        if (q.n_src || pre) {
            if (leader && q.n_src)
                inject_sources_dev(q.buf[cur], q.buf[cur ^ 1], q.src_off, q.wavelet, q.n_src,
                                   q.wl_len, q.step0 + ran, nullptr, nullptr, nullptr);
            if (!grid_barrier(q.bar, nb, a.budget_ns, a.status, &s_ok)) {
                ok = false;
                break;
            }
        }
        if constexpr (!kCells) {
            // default faces: the row-parallel body (one warp per row of 128 cells)
            step_rows<kC2F, TY>(a, q.tiles_x, false, threadIdx.y, blockIdx.x, nb);
        } else {
            for (uint32_t item = blockIdx.x; item < q.nitems; item += nb) {
                const uint32_t chunk = item / q.tiles, tile = item - chunk * q.tiles;
                const uint32_t zs = chunk * q.clen, ze = min(a.nz, zs + q.clen);
                zs_tile<kC2F, kCells, TY>(a, tile % q.tiles_x, tile / q.tiles_x, zs, ze);
            }
        }
        cur ^= 1;
        ++ran;
        const bool progress = (q.step0 + ran) % interval == 0;
        if (progress) {  // every CTA's writes of the step, then sum p^2
            double e = 0.0;
            if (!grid_barrier(q.bar, nb, a.budget_ns, a.status, &s_ok) ||
                !res_energy<TY>(r, q.buf[cur] + a.plane, &e, &s_ok)) {
                ok = false;
                break;
            }
            if (leader) L.energy = (float)e;
        }
        if (leader) {
            --L.steps_rem;
            ctrl->current_step = q.step0 + ran;
            ctrl->steps_remaining = L.steps_rem;
            ctrl->current_buffer = (uint32_t)cur;
            ctrl->steps_run = ran;
            if (progress) {
                ctrl->total_energy = L.energy;
                res_post(r, L.k2h_tail, L.k2h_head, L.dropped, 1u, 0u, q.step0 + ran, L.steps_rem,
                         L.energy, 0u);
            }
            decide(tail_hint);
        }
        ok = barrier_decision();  // end of the step: every CTA's writes, the decision
    }
    if (!ok) op = 0xFFu;
    // ---- leaving (persistent_fdtd.rs:942-978): final energy on TERMINATE
    if (op == kResExitTerm) {
        double e = 0.0;
        if (res_energy<TY>(r, q.buf[cur] + q.a.plane, &e, &s_ok)) {
            if (leader) L.energy = (float)e;
        } else {
            op = 0xFFu;
        }
    }
    if (leader) {
        ctrl->current_step = q.step0 + ran;
        ctrl->steps_remaining = L.steps_rem;
        ctrl->current_buffer = (uint32_t)cur;
        ctrl->steps_run = ran;
        ctrl->total_energy = L.energy;
        ctrl->messages_processed = L.msgs;
        ctrl->exit_reason = op == kResExitTerm ? 1u : (op == kResExitIdle ? 2u : 3u);
        if (op == kResExitTerm)
            res_post(r, L.k2h_tail, L.k2h_head, L.dropped, 3u, 0u, q.step0 + ran, 0u, L.energy, 0u);
        ctrl->k2h_dropped = L.dropped;
        __threadfence_system();
        ctrl->has_terminated = 1u;
    }
}

}  // namespace ws3d
