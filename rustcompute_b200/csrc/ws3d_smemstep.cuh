// ws3d_smemstep.cuh -- persistent steps with the field resident in shared
// memory (one GPU, default face layout, rows of at most 128 cells).
//
// For small grids (configuration c5: 128^3, 10,000 steps) a persistent step
// is latency-bound: every CTA reloads its cells and their neighbours from L2
// each step.  Here every CTA owns a block of whole rows -- all x, rows
// [y0, y0 + by), planes [z0, z0 + bz) -- and keeps p and p_prev of the block,
// with a one-cell halo in y and z, in shared memory for the whole launch.  A
// step reads only shared memory; the only global traffic per step is the
// block's four faces (first / last row of every plane, first / last plane)
// sent to the neighbours and theirs received into the halo:
//
//   step s: apply the sources of step s to the block and its halo copies
//           (each CTA from the global list, in source order: p += a, and
//           p_prev += a/2 on its own cells) -> compute p_{s+1} into the
//           p_prev slot (each cell reads its own p_prev only) -> store the
//           faces of p_{s+1} into the neighbours' exchange rows -> read the
//           neighbours' faces of p_{s+1} from this CTA's exchange rows into
//           the halo.
//
// Exchange rows hold 64-bit words (tag << 32 | value bits), stored and loaded
// as single relaxed 64-bit accesses, so a word that shows the expected tag
// also carries its value: no fence, no flag and no grid-wide barrier -- a
// CTA waits only for the words its halo needs (the scheme of NCCL's
// low-latency protocol).  Tags are tag0 + s + 1, increasing across launches
// (the host restarts them from a zeroed buffer before they wrap), so a word
// from an earlier step or launch never matches.  Rows alternate between two
// parities: a CTA stores the faces of step s+2 into the rows of step s only
// after it has received its neighbours' faces of step s+1, which they store
// after reading the faces of step s.  After the last step each CTA writes its
// block of p_n to buf[n & 1] and of p_{n-1} to buf[(n - 1) & 1] -- the roles
// k_persistent leaves -- so the fields are bit-identical to per-step launches
// (cell_rule<false>, the reference operation order).
//
// Halo cells outside the grid (y = -1 / H, z = -1 / D) and the x halo (x = -1
// and x = pitch, outside every row) stay zero; the cells next to them are
// faces, whose rule reads none of their neighbours.  Every wait for a tagged
// word is bounded, and gives up at once when another CTA recorded an error.
#pragma once

#include "ws3d_persistent.cuh"

namespace ws3d {

constexpr int kSmemThreads = 1024;       // 32 warps: one warp per row slot
constexpr int kSmemMaxBytes = 220 * 1024;

struct SmemArgs {
    StepParams a;                        // geometry and constants
    float* buf[2];                       // plane -1 of the two field buffers (pressure, prev)
    unsigned long long* xch;             // exchange rows: [parity][block][2 (by + bz)][pitch]
    uint32_t tag0;                       // faces of step s carry tag tag0 + s + 1
    const uint64_t* src_off;             // (z+1) * plane + y * pitch + x
    const float* wavelet;
    uint32_t n_src;
    uint64_t wl_len;
    uint64_t step0;
    uint64_t nsteps;
    uint32_t by, bz, yblocks, zblocks;   // block shape, blocks along y and z
};

__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait for the word at p to carry `tag` (high 32 bits); returns the
// word.  On a give-up (budget spent: status bit 3; or another CTA already
// recorded an error) *ok = 0 and the value is meaningless.
__device__ __noinline__ unsigned long long smem_tag_wait(const unsigned long long* p,
                                                         unsigned long long tag,
                                                         unsigned long long budget_ns,
                                                         unsigned int* status, int* ok) {
    const unsigned long long t0 = global_ns();
    for (unsigned int it = 0; it < (1u << 26); ++it) {
        const unsigned long long v = ld_relaxed_gpu_u64(p);
        if ((v & 0xffffffff00000000ull) == tag) return v;
        if ((it & 63u) == 63u) {
            if (*reinterpret_cast<volatile unsigned int*>(status) != 0u) {
                *ok = 0;
                return 0;
            }
            if (global_ns() - t0 > budget_ns) break;
        }
    }
    atomicOr(status, 8u);
    *ok = 0;
    return 0;
}

template <bool kC2F>
__global__ void __launch_bounds__(kSmemThreads, 1) k_persistent_smem(SmemArgs q) {
    extern __shared__ float sm[];
    const StepParams& a = q.a;
    const uint32_t pitch = a.pitch;
    const int SX = (int)pitch + 2, SY = (int)q.by + 2;
    const int SP = SX * SY;                       // one shared plane
    const int SV = SP * ((int)q.bz + 2);          // one shared volume
    // volume k & 1 holds p_s at step s = k, the other one p_{s-1}
    float* c2s = sm + 2 * SV;                     // kC2F: pitch x by x bz
    const uint32_t yb = blockIdx.x % q.yblocks, zb = blockIdx.x / q.yblocks;
    const uint32_t y0 = yb * q.by, z0 = zb * q.bz;
    const uint32_t ny = min(q.by, a.H - y0), nzb = min(q.bz, a.nz - z0);
    const int64_t P = (int64_t)a.plane;
    const int t = threadIdx.x;
    const size_t nblk = gridDim.x, R = smem_xch_rows(q.by, q.bz);
    auto sidx = [&](int x, int y, int z) { return (z + 1) * SP + (y + 1) * SX + (x + 1); };
    auto gofs = [&](uint32_t x, uint32_t y, uint32_t z) {  // from plane -1
        return (int64_t)(z + 1) * P + (int64_t)y * pitch + x;
    };

    // ---- load p with its y / z halo, p_prev and c2 of the block
    for (int i = t; i < 2 * SV; i += kSmemThreads) sm[i] = 0.f;
    __syncthreads();
    {
        const float* p0 = q.buf[0];
        const float* pp0 = q.buf[1];
        const int rows = (int)(nzb + 2) * (int)(ny + 2);
        for (int r = t >> 5; r < rows; r += kSmemThreads / 32) {
            const int zz = r / (int)(ny + 2) - 1, yy = r % (int)(ny + 2) - 1;
            const int64_t gz = (int64_t)z0 + zz, gy = (int64_t)y0 + yy;
            if (gz < 0 || gz >= (int64_t)a.nz || gy < 0 || gy >= (int64_t)a.H) continue;
            const bool own = zz >= 0 && zz < (int)nzb && yy >= 0 && yy < (int)ny;
            for (uint32_t x = threadIdx.x & 31u; x < pitch; x += 32) {
                const int64_t g = gofs(x, (uint32_t)gy, (uint32_t)gz);
                sm[sidx((int)x, yy, zz)] = __ldcg(p0 + g);
                if (own) {
                    sm[SV + sidx((int)x, yy, zz)] = __ldcg(pp0 + g);
                    if (kC2F)
                        c2s[((size_t)zz * q.by + yy) * pitch + x] = __ldg(a.c2f + g - P);
                }
            }
        }
    }
    __syncthreads();

    const int warp = t >> 5, lane = t & 31;
    for (uint64_t s = 0; s < q.nsteps; ++s) {
        float* pc = sm + (s & 1) * SV;          // p_s
        float* pv = sm + ((s & 1) ^ 1) * SV;    // p_{s-1}, becomes p_{s+1}
        // sources of this step, in order (one thread: coinciding sources add in turn)
        if (q.n_src && t == 0) {
            const uint64_t st = q.step0 + s;
            for (uint32_t k = 0; k < q.n_src; ++k) {
                const uint64_t off = q.src_off[k];
                const int64_t gz = (int64_t)(off / (uint64_t)P) - 1;
                const uint64_t rem = off - (uint64_t)(gz + 1) * (uint64_t)P;
                const int64_t gy = (int64_t)(rem / pitch), gx = (int64_t)(rem - gy * pitch);
                const int zz = (int)(gz - z0), yy = (int)(gy - y0);
                if (zz < -1 || zz > (int)nzb || yy < -1 || yy > (int)ny) continue;
                const float amp = st < q.wl_len ? q.wavelet[(uint64_t)k * q.wl_len + st] : 0.0f;
                const int i = sidx((int)gx, yy, zz);
                pc[i] = __fadd_rn(pc[i], amp);
                if (zz >= 0 && zz < (int)nzb && yy >= 0 && yy < (int)ny)
                    pv[i] = __fadd_rn(pv[i], __fmul_rn(amp, 0.5f));
            }
        }
        if (q.n_src) __syncthreads();

        // ---- p_{s+1} on the block: a warp takes (row, 32-column chunk) pairs
        // and sweeps their z column, lanes along x
        const int xch = (int)pitch / 32;
        for (int pr = warp; pr < (int)ny * xch; pr += kSmemThreads / 32) {
            const int y = pr / xch;
            const uint32_t gy = y0 + (uint32_t)y;
            {
                const uint32_t x = (uint32_t)((pr - y * xch) * 32 + lane);
                float dn = pc[sidx((int)x, y, -1)];
                float c = pc[sidx((int)x, y, 0)];
                for (int z = 0; z < (int)nzb; ++z) {
                    const int i = sidx((int)x, y, z);
                    const float up = pc[i + SP];
                    const uint32_t gz = a.z0 + z0 + (uint32_t)z;
                    const float c2 = kC2F ? c2s[((size_t)z * q.by + y) * pitch + x] : a.c2;
                    pv[i] = cell_rule<false>(x, gy, gz, is_interior(x, gy, gz, a), pc[i - 1],
                                             pc[i + 1], pc[i - SX], pc[i + SX], dn, up, c, pv[i],
                                             c2, 0, 0.f, a);
                    dn = c;
                    c = up;
                }
            }
        }
        __syncthreads();

        // ---- faces of p_{s+1} into the neighbours' exchange rows, then theirs
        // into the halo: 64-bit words of (tag << 32 | value bits), so a word
        // read with the expected tag carries its value -- no fence, no flag
        const bool last = s + 1 == q.nsteps;
        if (!last) {
            const uint32_t par = (uint32_t)((s + 1) & 1);
            const unsigned long long tag = (unsigned long long)(q.tag0 + (uint32_t)s + 1u) << 32;
            const int rows = 2 * (int)nzb + 2 * (int)ny;
            for (int r = warp; r < rows; r += kSmemThreads / 32) {
                int yy, zz, kind;
                if (r < 2 * (int)nzb) {
                    zz = r >> 1;
                    kind = r & 1;
                    yy = kind ? (int)ny - 1 : 0;
                } else {
                    yy = (r - 2 * (int)nzb) >> 1;
                    kind = 2 + ((r - 2 * (int)nzb) & 1);
                    zz = kind == 3 ? (int)nzb - 1 : 0;
                }
                uint32_t nbk;
                int side, i;
                if (!smem_face_dest(blockIdx.x, q.yblocks, q.zblocks, kind, yy, zz, &nbk, &side, &i))
                    continue;
                unsigned long long* dst =
                    q.xch + (((size_t)par * nblk + nbk) * R + smem_xch_slot(q.by, q.bz, side, i)) * pitch;
                const float* src = pv + sidx(0, yy, zz);
                for (uint32_t x = (uint32_t)lane; x < pitch; x += 32)
                    st_relaxed_gpu_u64(dst + x, tag | __float_as_uint(src[x]));
            }
            // the halo: rows y0 - 1 / y0 + ny of every plane, planes z0 - 1 / z0 + nzb
            int ok = 1;
            for (int r = warp; r < rows && ok; r += kSmemThreads / 32) {
                int yy, zz, side, i;
                bool have;
                if (r < 2 * (int)nzb) {
                    zz = r >> 1;
                    side = r & 1;
                    yy = side ? (int)ny : -1;
                    i = zz;
                    have = side ? yb + 1 < q.yblocks : yb > 0;
                } else {
                    yy = (r - 2 * (int)nzb) >> 1;
                    side = 2 + ((r - 2 * (int)nzb) & 1);
                    zz = side == 3 ? (int)nzb : -1;
                    i = yy;
                    have = side == 3 ? zb + 1 < q.zblocks : zb > 0;
                }
                if (!have) continue;
                const unsigned long long* srcw =
                    q.xch + (((size_t)par * nblk + blockIdx.x) * R + smem_xch_slot(q.by, q.bz, side, i)) * pitch;
                // all of this lane's words in flight at once (rows are at most
                // 128 cells: four per lane), then the tags
                unsigned long long v[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t x = (uint32_t)lane + 32u * k;
                    v[k] = x < pitch ? ld_relaxed_gpu_u64(srcw + x) : tag;
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t x = (uint32_t)lane + 32u * k;
                    if (x >= pitch) continue;
                    if ((v[k] & 0xffffffff00000000ull) != tag)
                        v[k] = smem_tag_wait(srcw + x, tag, a.budget_ns, a.status, &ok);
                    pv[sidx((int)x, yy, zz)] = __uint_as_float((uint32_t)v[k]);
                }
            }
            if (!__syncthreads_and(ok)) return;
        }
    }

    // ---- the block of p_n and p_{n-1} into the roles the host expects
    const uint64_t n = q.nsteps;
    const float* pn = sm + (n & 1) * SV;
    const float* pn1 = sm + ((n & 1) ^ 1) * SV;
    float* gp = q.buf[n & 1];
    float* gpp = q.buf[(n & 1) ^ 1];
    const int rows = (int)nzb * (int)ny;
    for (int r = warp; r < rows; r += kSmemThreads / 32) {
        const int zz = r / (int)ny, yy = r % (int)ny;
        for (uint32_t x = (uint32_t)lane; x < pitch; x += 32) {
            const int64_t g = gofs(x, y0 + (uint32_t)yy, z0 + (uint32_t)zz);
            gp[g] = pn[sidx((int)x, yy, zz)];
            gpp[g] = pn1[sidx((int)x, yy, zz)];
        }
    }
}

}  // namespace ws3d
