// ws3d_index.h -- address arithmetic of the step kernels, shared by the device
// code and by a host-side bounds check (tests/index_check.cpp), which walks
// every CTA, thread and plane of a launch and verifies that each load and
// store the kernel issues stays inside the slab allocation.
//
// All offsets are signed 64-bit element offsets relative to owned plane 0 of
// a slab (ghost plane -1 starts at -plane).  Every intermediate is widened to
// int64 before subtraction, so no unsigned wrap-around can occur.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define WS3D_HD __host__ __device__ __forceinline__
#else
#define WS3D_HD inline
#endif

namespace ws3d {

constexpr int kZsTileX = 128;  // cells per CTA row (32 lanes x float4)

// Two-step kernel (k_step_tma2): tile height in rows and co-resident CTAs per
// SM.  TY + 2 consumer warps (one extended row each) plus one producer warp
// per CTA; a tile of 16 rows takes one CTA of 19 warps per SM (shared memory),
// a tile of 8 rows two CTAs of 11 warps.  Measured on B200 (C3 512^3 / C4
// 1024^3, 4 stages): 16 rows 514 / 4122 us per launch, 8 rows (2 CTAs, 5
// stages) 568 / 4753 us -- half the halo rows and halo columns per core cell,
// and 96 registers without spills instead of 80 with spills.
#ifndef WS3D_TB_TY
#define WS3D_TB_TY 16
#endif
constexpr int kTbTY = WS3D_TB_TY;
constexpr int kTbCtasPerSm = kTbTY >= 16 ? 1 : 2;
static_assert(kTbTY % 2 == 0 && kTbTY >= 8 && kTbTY <= 28, "two-step tile height");

// Per-thread constants of the z-streaming kernel.
struct ZsLane {
    int64_t row;    // offset of this thread's float4 inside a plane
    int64_t rowlo;  // halo row y0-1 (valid when ylo)
    int64_t rowhi;  // halo row y0+TY (valid when yhi)
    int64_t offxl;  // halo float x0-1 (valid when xl)
    int64_t offxr;  // halo float x0+128 (valid when xr)
    uint32_t x, y, x0, y0;
    bool act, ylo, yhi, xl, xr;
};

template <int TY>
WS3D_HD ZsLane zs_lane(uint32_t bx, uint32_t by, int lane, int w, uint32_t W, uint32_t H,
                       uint32_t pitch) {
    ZsLane L;
    L.x0 = bx * (uint32_t)kZsTileX;
    L.x = L.x0 + 4u * (uint32_t)lane;
    L.y0 = by * (uint32_t)TY;
    L.y = L.y0 + (uint32_t)w;
    const bool xin = L.x < pitch;
    const bool yin = L.y < H;
    L.act = xin && yin;
    L.ylo = (w == 0) && (L.y0 > 0) && xin;
    L.yhi = (w == TY - 1) && (L.y0 + (uint32_t)TY < H) && xin;
    L.xl = (lane == 0) && (L.x0 > 0) && yin;
    L.xr = (lane == 31) && (L.x0 + (uint32_t)kZsTileX < W) && yin;
    const int64_t P = (int64_t)pitch;
    L.row = (int64_t)L.y * P + (int64_t)L.x;
    L.rowlo = ((int64_t)L.y0 - 1) * P + (int64_t)L.x;
    L.rowhi = ((int64_t)L.y0 + TY) * P + (int64_t)L.x;
    L.offxl = (int64_t)L.y * P + (int64_t)L.x0 - 1;
    L.offxr = (int64_t)L.y * P + (int64_t)L.x0 + kZsTileX;
    return L;
}

// Offset of plane `z` (may be -1 or nz: the ghosts).
WS3D_HD int64_t zs_plane(int64_t z, int64_t plane) { return z * plane; }

// Persistent steps with the field in shared memory (k_persistent_smem): bytes
// of one CTA's block (p and p_prev with a one-cell halo, c2 of its own cells)
// and the block shape: the fewest cells per CTA such that every block is
// co-resident (at most `max_blocks`, one per SM) and fits `max_bytes`, then
// the fewest face rows (by + bz).  Returns false when no shape qualifies.
WS3D_HD uint64_t smem_step_bytes(uint32_t pitch, uint32_t by, uint32_t bz, bool c2f) {
    const uint64_t vol = (uint64_t)(pitch + 2) * (by + 2) * (bz + 2);
    return 2 * vol * 4 + (c2f ? (uint64_t)pitch * by * bz * 4 : 0);
}
WS3D_HD bool smem_step_shape(uint32_t pitch, uint32_t H, uint32_t nz, uint32_t max_blocks,
                             bool c2f, uint64_t max_bytes, uint32_t* by, uint32_t* bz) {
    *by = *bz = 0;
    uint64_t best_cells = ~0ull, best_face = ~0ull;
    for (uint32_t cy = 1; cy <= 128; cy *= 2)
        for (uint32_t cz = 1; cz <= 128; cz *= 2) {
            if (smem_step_bytes(pitch, cy, cz, c2f) > max_bytes) continue;
            const uint64_t nblk = (uint64_t)((H + cy - 1) / cy) * (uint64_t)((nz + cz - 1) / cz);
            if (nblk > max_blocks) continue;
            const uint64_t cells = (uint64_t)cy * cz, face = cy + cz;
            if (cells < best_cells || (cells == best_cells && face < best_face)) {
                best_cells = cells;
                best_face = face;
                *by = cy;
                *bz = cz;
            }
        }
    return *by != 0;
}

// Face exchange of k_persistent_smem.  Block b receives its halo faces in
// 2 * (by + bz) rows of pitch tagged words of its own: rows [0, bz) the
// y-halo row below (row -1) of planes 0..bz-1, [bz, 2bz) the y-halo row above
// (row ny), [2bz, 2bz + by) the z-halo plane below (plane -1) of rows
// 0..by-1, [2bz + by, 2bz + 2by) the plane above (plane nzb).  side: 0 below
// in y, 1 above in y, 2 below in z, 3 above in z; i: the plane (sides 0, 1)
// or the row (sides 2, 3).
WS3D_HD uint32_t smem_xch_rows(uint32_t by, uint32_t bz) { return 2u * (by + bz); }
WS3D_HD uint32_t smem_xch_slot(uint32_t by, uint32_t bz, int side, int i) {
    return side == 0 ? (uint32_t)i
         : side == 1 ? bz + (uint32_t)i
         : side == 2 ? 2u * bz + (uint32_t)i
                     : 2u * bz + by + (uint32_t)i;
}
// Where face row (yy, zz) of block b goes.  kind 0: row 0 of plane zz (to the
// block below in y, which holds it as its halo above); 1: the last row (block
// above, halo below); 2: plane 0 (block below in z, halo above); 3: the last
// plane (block above in z, halo below).  Blocks are numbered zb * yblocks +
// yb.  False when there is no neighbour on that side.
WS3D_HD bool smem_face_dest(uint32_t b, uint32_t yblocks, uint32_t zblocks, int kind, int yy,
                            int zz, uint32_t* nb, int* side, int* i) {
    const uint32_t yb = b % yblocks, zb = b / yblocks;
    if (kind == 0) {
        if (yb == 0) return false;
        *nb = b - 1;
        *side = 1;
        *i = zz;
    } else if (kind == 1) {
        if (yb + 1 >= yblocks) return false;
        *nb = b + 1;
        *side = 0;
        *i = zz;
    } else if (kind == 2) {
        if (zb == 0) return false;
        *nb = b - yblocks;
        *side = 3;
        *i = yy;
    } else {
        if (zb + 1 >= zblocks) return false;
        *nb = b + yblocks;
        *side = 2;
        *i = yy;
    }
    return true;
}

// Block-parallel persistent body (k_persistent_rows, k_resident): block b of
// a step is x-tile tx of rows yb*NW .. yb*NW + NW - 1 of plane z (one warp per
// row, 128 cells a row).  On z-slabs the interior planes 1 .. nz-2 come first,
// then plane 0, then plane nz-1 (their waits for the neighbours' flags overlap
// the interior blocks).
struct RowCoord {
    uint32_t z, yb, tx;
};
WS3D_HD RowCoord row_coord(uint64_t b, uint32_t yblocks, uint32_t tiles_x, uint32_t nz, bool slab) {
    const uint64_t per_plane = (uint64_t)yblocks * tiles_x;
    const uint64_t k = b / per_plane;
    const uint32_t rem = (uint32_t)(b - k * per_plane);
    RowCoord c;
    c.z = (uint32_t)k;
    if (slab && nz > 1) c.z = k + 2 < nz ? (uint32_t)k + 1u : (k + 2 == nz ? 0u : nz - 1);
    c.yb = rem / tiles_x;
    c.tx = rem - c.yb * tiles_x;
    return c;
}

// Order in which z-chunks are assigned to blockIdx.z.  With a halo exchange,
// chunk 0 and the last chunk (the ones that wait for a neighbour) go last.
WS3D_HD uint32_t zs_chunk_order(uint32_t bz, uint32_t gz, bool halo) {
    return (halo && gz > 1) ? (bz + 1) % gz : bz;
}

// z-range of CTA `bz`: [zb, ze), empty when zb >= nz.
WS3D_HD void zs_chunk(uint32_t bz, uint32_t zchunk, uint32_t nz, uint32_t* zb, uint32_t* ze) {
    const uint64_t b = (uint64_t)bz * zchunk;
    *zb = b < nz ? (uint32_t)b : nz;
    const uint64_t e = b + zchunk;
    *ze = e < nz ? (uint32_t)e : nz;
}

// Launch geometry of the z-streaming kernel (host side): enough CTAs for ~8
// resident waves over the SMs.  Each chunk re-reads two extra planes, so
// chunks stay >= 16 planes when the slab streams from HBM; a slab whose
// three fields fit in L2 (<= 64 MiB) uses chunks down to 4 planes, since
// there the re-reads are L2 hits and the per-plane latency dominates.
template <int TY>
inline uint32_t zs_zchunk(uint32_t pitch, uint32_t H, uint32_t nz, int sm_count) {
    const uint32_t tiles = ((pitch + kZsTileX - 1) / kZsTileX) * ((H + TY - 1) / TY);
    const uint32_t want = (uint32_t)(sm_count > 0 ? sm_count : 1) * 3u * 8u;
    uint32_t nchunks = (want + tiles - 1) / tiles;
    if (nchunks < 1) nchunks = 1;
    uint32_t chunk = (nz + nchunks - 1) / nchunks;
    const uint64_t field_bytes = (uint64_t)pitch * H * nz * 4u * 3u;
    const uint32_t min_chunk = field_bytes <= (64ull << 20) ? 4u : 16u;
    if (chunk < min_chunk) chunk = min_chunk;
    const uint32_t cap = nz > 0 ? nz : 1;
    return chunk < cap ? chunk : cap;
}

template <int TY>
inline void zs_grid(uint32_t pitch, uint32_t H, uint32_t nz, uint32_t zchunk, uint32_t* gx,
                    uint32_t* gy, uint32_t* gz) {
    *gx = (pitch + kZsTileX - 1) / kZsTileX;
    *gy = (H + TY - 1) / TY;
    *gz = (nz + zchunk - 1) / zchunk;
}

// Schedule of the TMA kernel: (grid, chunk length, items) for `tiles` tiles
// of nz planes on `resident` co-resident CTAs.  z is cut into chunks of at
// least `min_chunk` planes (whole columns when nz < 2 * min_chunk); the chunk count maximises the
// use of the resident CTA slots, items / (rounds * resident), preferring
// fewer chunks on ties (fewer re-read boundary planes).
struct TmaSchedule {
    uint32_t grid, clen, nitems;
};
inline TmaSchedule tma_schedule(uint32_t tiles, uint32_t nz, uint32_t resident,
                                uint32_t min_chunk = 32) {
    TmaSchedule s;
    if (resident < 1) resident = 1;
    if (tiles < 1) tiles = 1;
    if (min_chunk < 1) min_chunk = 1;
    uint32_t best_k = 1;
    double best = -1.0;
    const uint32_t kmax = nz / min_chunk > 1 ? nz / min_chunk : 1;
    for (uint32_t k = 1; k <= kmax && k <= 1024; ++k) {
        const uint32_t clen = (nz + k - 1) / k;
        const uint32_t chunks = (nz + clen - 1) / clen;
        const uint64_t items = (uint64_t)chunks * tiles;
        const uint64_t rounds = (items + resident - 1) / resident;
        const double use = (double)items / ((double)rounds * resident);
        if (use > best + 1e-9) {
            best = use;
            best_k = k;
        }
    }
    s.clen = (nz + best_k - 1) / best_k;
    if (s.clen < 1) s.clen = 1;
    const uint32_t chunks = (nz + s.clen - 1) / s.clen;
    s.nitems = chunks * tiles;
    s.grid = s.nitems < resident ? s.nitems : resident;
    return s;
}

// Schedule of the two-step kernel: every run of clen planes costs clen + 4
// staged items (two planes of X beyond the run, two leading pressure planes),
// so pick the chunk count that minimises rounds x (clen + 4) -- fewer, longer
// runs unless the last round leaves too many CTAs idle.
inline TmaSchedule tb_schedule(uint32_t tiles, uint32_t nz, uint32_t resident,
                               uint32_t min_chunk = 16) {
    TmaSchedule s;
    if (resident < 1) resident = 1;
    if (tiles < 1) tiles = 1;
    if (min_chunk < 1) min_chunk = 1;
    uint32_t best_k = 1;
    uint64_t best = ~0ull;
    const uint32_t kmax = nz / min_chunk > 1 ? nz / min_chunk : 1;
    for (uint32_t k = 1; k <= kmax && k <= 1024; ++k) {
        const uint32_t clen = (nz + k - 1) / k;
        const uint32_t chunks = (nz + clen - 1) / clen;
        const uint64_t items = (uint64_t)chunks * tiles;
        const uint64_t rounds = (items + resident - 1) / resident;
        const uint64_t cost = rounds * (clen + 4u);
        if (cost < best) {
            best = cost;
            best_k = k;
        }
    }
    s.clen = (nz + best_k - 1) / best_k;
    if (s.clen < 1) s.clen = 1;
    const uint32_t chunks = (nz + s.clen - 1) / s.clen;
    s.nitems = chunks * tiles;
    s.grid = s.nitems < resident ? s.nitems : resident;
    return s;
}

// ---- cp.async pipeline (k_step_async): per-thread copy assignments --------
// A stage holds the front pressure plane as 10 rows x 136 floats (x from
// x0-4, rows y0-1 .. y0+8) = 340 float4 chunks, and p_prev / c2 as 8 x 128
// floats = 256 float4 chunks each.  Thread t of 256 copies P chunks t and
// t + 256 (< 340) and chunk t of p_prev and c2.  Chunks outside the grid are
// zero-filled (no global access).
constexpr int kAsyncTY = 8;
constexpr int kAsyncPRow = 136;
constexpr int kAsyncPChunks = kAsyncPRow / 4 * (kAsyncTY + 2);  // 340

struct AsyncChunk {
    bool valid;       // inside the grid: copy from global, else zero-fill
    int64_t goff;     // in-plane global element offset (valid only)
    int32_t soff;     // shared-memory element offset inside the tile
};

WS3D_HD AsyncChunk async_p_chunk(int c, uint32_t x0, uint32_t y0, uint32_t H, uint32_t pitch) {
    AsyncChunk a;
    const int r = c / (kAsyncPRow / 4), q = c - r * (kAsyncPRow / 4);
    const int64_t y = (int64_t)y0 - 1 + r;
    const int64_t x = (int64_t)x0 - 4 + 4 * q;
    a.valid = y >= 0 && y < (int64_t)H && x >= 0 && x < (int64_t)pitch;
    a.goff = a.valid ? y * (int64_t)pitch + x : 0;
    a.soff = r * kAsyncPRow + 4 * q;
    return a;
}

WS3D_HD AsyncChunk async_t_chunk(int c, uint32_t x0, uint32_t y0, uint32_t H, uint32_t pitch) {
    AsyncChunk a;
    const int r = c / 32, q = c - r * 32;
    const int64_t y = (int64_t)y0 + r;
    const int64_t x = (int64_t)x0 + 4 * q;
    a.valid = y < (int64_t)H && x < (int64_t)pitch;
    a.goff = a.valid ? y * (int64_t)pitch + x : 0;
    a.soff = r * 128 + 4 * q;
    return a;
}

// Item order for slabs: boundary z-chunks (the ones that wait for a
// neighbour) after all interior chunks.
WS3D_HD uint32_t async_chunk_of(uint32_t item, uint32_t tiles, uint32_t nchunks, bool halo) {
    const uint32_t c = item / tiles;
    return (halo && nchunks > 1) ? (c + 1) % nchunks : c;
}

}  // namespace ws3d
