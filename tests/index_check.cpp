// Host-side bounds check of the z-streaming kernel's addressing.
//
// Replays, for every CTA (or for the corner CTAs of very large launches),
// every thread and every plane, the loads and stores k_step_zstream issues,
// using the same helpers (rustcompute_b200/csrc/ws3d_index.h), and verifies
// that each access lies inside its allocation, is 16-byte aligned for float4
// accesses and does not straddle a row.  Exit code 0 = all accesses in bounds.
//
// Usage: index_check W H nz sm_count [TY [halo [kernel: 0 zstream, 1 async, 2 rows]]]
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "ws3d_index.h"

using namespace ws3d;

static long long g_checked = 0;
static int g_bad = 0;

struct Field {
    const char* name;
    bool ghosts;  // p: ghost planes -1 and nz are readable
};

static void check(const Field& f, int64_t o, int n, uint32_t pitch, uint32_t nz, int64_t plane,
                  const char* what, uint32_t bx, uint32_t by, uint32_t bz, int lane, int w) {
    ++g_checked;
    const int64_t lo = f.ghosts ? -plane : 0;
    const int64_t hi = f.ghosts ? (int64_t)(nz + 1) * plane : (int64_t)nz * plane;
    int64_t in_row = ((o % (int64_t)pitch) + pitch) % (int64_t)pitch;
    bool ok = o >= lo && o + n <= hi && in_row + n <= (int64_t)pitch;
    if (n == 4 && (o % 4) != 0) ok = false;
    if (!ok && g_bad < 20) {
        fprintf(stderr, "OUT OF BOUNDS %s %s: off=%lld n=%d [%lld,%lld) block=(%u,%u,%u) lane=%d w=%d\n",
                f.name, what, (long long)o, n, (long long)lo, (long long)hi, bx, by, bz, lane, w);
    }
    if (!ok) ++g_bad;
}

template <int TY>
static void run(uint32_t W, uint32_t H, uint32_t nz, int sms, bool halo) {
    const uint32_t pitch = (W + 31u) & ~31u;
    const int64_t P = (int64_t)H * pitch;
    const uint32_t chunk = zs_zchunk<TY>(pitch, H, nz, sms);
    uint32_t gx, gy, gz;
    zs_grid<TY>(pitch, H, nz, chunk, &gx, &gy, &gz);
    const Field fp{"p", true}, fpp{"pp", false}, fc2{"c2", false}, fty{"types", false},
        frf{"refl", false};
    const bool sample = (uint64_t)gx * gy * gz * 32 * TY * (chunk + 2) > 30000000ull;
    auto pick = [&](uint32_t n) {
        std::vector<uint32_t> v;
        if (!sample || n <= 4) {
            for (uint32_t i = 0; i < n; ++i) v.push_back(i);
        } else {
            v = {0, 1, n / 2, n - 2, n - 1};
        }
        return v;
    };
    for (uint32_t bz : pick(gz))
        for (uint32_t by : pick(gy))
            for (uint32_t bx : pick(gx)) {
                uint32_t zb, ze;
                zs_chunk(zs_chunk_order(bz, gz, halo), chunk, nz, &zb, &ze);
                if (zb >= ze) continue;
                for (int w = 0; w < TY; ++w)
                    for (int lane = 0; lane < 32; ++lane) {
                        const ZsLane L = zs_lane<TY>(bx, by, lane, w, W, H, pitch);
                        auto C = [&](const Field& f, int64_t z, int64_t off, int n, const char* what) {
                            check(f, zs_plane(z, P) + off, n, pitch, nz, P, what, bx, by, bz, lane, w);
                        };
                        if (L.act) {
                            C(fp, (int64_t)zb - 1, L.row, 4, "prologue pm");
                            C(fp, zb, L.row, 4, "prologue pc");
                        }
                        if (L.ylo) C(fp, zb, L.rowlo, 4, "prologue ylo");
                        if (L.yhi) C(fp, zb, L.rowhi, 4, "prologue yhi");
                        if (L.xl) C(fp, zb, L.offxl, 1, "prologue xl");
                        if (L.xr) C(fp, zb, L.offxr, 1, "prologue xr");
                        if (L.act) {
                            C(fp, (int64_t)zb + 1, L.row, 4, "prologue pn");
                            C(fpp, zb, L.row, 4, "prologue pp");
                            C(fc2, zb, L.row, 4, "prologue c2");
                            C(fty, zb, L.row, 4, "prologue types");
                        }
                        for (uint32_t zl = zb; zl < ze; ++zl) {
                            const bool more = zl + 1 < ze;
                            if (more) {
                                if (L.act) {
                                    C(fp, (int64_t)zl + 2, L.row, 4, "loop pn2");
                                    C(fpp, (int64_t)zl + 1, L.row, 4, "loop pp");
                                    C(fc2, (int64_t)zl + 1, L.row, 4, "loop c2");
                                    C(fty, (int64_t)zl + 1, L.row, 4, "loop types");
                                }
                                if (L.ylo) C(fp, (int64_t)zl + 1, L.rowlo, 4, "loop ylo");
                                else if (L.yhi) C(fp, (int64_t)zl + 1, L.rowhi, 4, "loop yhi");
                                if (L.xl) C(fp, (int64_t)zl + 1, L.offxl, 1, "loop xl");
                                else if (L.xr) C(fp, (int64_t)zl + 1, L.offxr, 1, "loop xr");
                            }
                            if (L.act) {
                                for (int k = 0; k < 4; ++k) C(frf, zl, L.row + k, 1, "refl");
                                C(fpp, zl, L.row, 4, "store");
                                // peer stores into a neighbour's ghost plane (one plane)
                                if (halo && (zl == 0 || zl + 1 == nz)) {
                                    ++g_checked;
                                    if (!(L.row >= 0 && L.row + 4 <= P && L.row % 4 == 0)) {
                                        ++g_bad;
                                        fprintf(stderr, "OUT OF BOUNDS peer store row=%lld\n",
                                                (long long)L.row);
                                    }
                                }
                            }
                        }
                    }
            }
}

// The cp.async kernel: replay every CTA's issue sequence (P / p_prev / c2
// chunk copies of each stage-item) and its consumer's global loads / stores.
static void run_async(uint32_t W, uint32_t H, uint32_t nz, int sms, bool halo) {
    const uint32_t pitch = (W + 31u) & ~31u;
    const int64_t P = (int64_t)H * pitch;
    const uint32_t tiles_x = (pitch + 127) / 128;
    const uint32_t tiles = tiles_x * ((H + kAsyncTY - 1) / kAsyncTY);
    const uint32_t resident = (uint32_t)(sms > 0 ? sms : 1) * 3u;
    const uint64_t field_bytes = (uint64_t)P * nz * 12u;
    const TmaSchedule sch = tma_schedule(tiles, nz, resident, field_bytes <= (64ull << 20) ? 8u : 32u);
    const uint32_t nchunks = (nz + sch.clen - 1) / sch.clen;
    const Field fp{"p", true}, fpp{"pp", false}, fc2{"c2", false};
    uint64_t covered = 0;
    for (uint32_t b = 0; b < sch.grid; ++b) {
        for (uint32_t item = b; item < sch.nitems; item += sch.grid) {
            const uint32_t chunk = async_chunk_of(item, tiles, nchunks, halo);
            const uint32_t tile = item % tiles;
            const uint32_t zs = chunk * sch.clen, ze = zs + sch.clen < nz ? zs + sch.clen : nz;
            covered += (uint64_t)(ze - zs);
            const uint32_t x0 = (tile % tiles_x) * 128u, y0 = (tile / tiles_x) * kAsyncTY;
            for (uint32_t i = 0; i <= ze - zs; ++i) {
                for (int t = 0; t < 32 * kAsyncTY; ++t) {
                    for (int c = t; c < kAsyncPChunks; c += 32 * kAsyncTY) {
                        const AsyncChunk ch = async_p_chunk(c, x0, y0, H, pitch);
                        if (ch.valid)
                            check(fp, zs_plane((int64_t)zs + i, P) + ch.goff, 4, pitch, nz, P,
                                  "async P copy", b, 0, 0, t, 0);
                    }
                    if (i > 0) {
                        const AsyncChunk ch = async_t_chunk(t, x0, y0, H, pitch);
                        if (ch.valid) {
                            check(fpp, zs_plane((int64_t)zs + i - 1, P) + ch.goff, 4, pitch, nz,
                                  P, "async pp copy", b, 0, 0, t, 0);
                            check(fc2, zs_plane((int64_t)zs + i - 1, P) + ch.goff, 4, pitch, nz,
                                  P, "async c2 copy", b, 0, 0, t, 0);
                        }
                    }
                }
            }
            for (int w = 0; w < kAsyncTY; ++w)
                for (int lane = 0; lane < 32; ++lane) {
                    const uint32_t x = x0 + 4u * lane, y = y0 + w;
                    if (!(x < pitch && y < H)) continue;
                    const int64_t row = (int64_t)y * pitch + x;
                    check(fp, zs_plane((int64_t)zs - 1, P) + row, 4, pitch, nz, P, "async pm", b,
                          0, 0, lane, w);
                    for (uint32_t z = zs; z < ze; ++z)
                        check(fpp, zs_plane(z, P) + row, 4, pitch, nz, P, "async store", b, 0, 0,
                              lane, w);
                }
        }
    }
    if (covered != (uint64_t)tiles * nz) {
        ++g_bad;
        fprintf(stderr, "async schedule covers %llu plane-tiles, expected %llu\n",
                (unsigned long long)covered, (unsigned long long)tiles * nz);
    }
}

// k_persistent_rows / k_resident's block body: every block of one step
// (row_coord, the kernels' own mapping), every warp row and lane: the four or
// five float4 loads of its own row, the block's two halo rows, the two x-halo
// loads, the store and the z-slab peer stores; every float4 of the owned
// planes written exactly once.
static void run_rows(uint32_t W, uint32_t H, uint32_t nz, bool slab, int NW) {
    const uint32_t pitch = (W + 31u) & ~31u;
    const int64_t P = (int64_t)H * pitch;
    const uint32_t tiles_x = (pitch + 127u) / 128u;
    const uint32_t yblocks = (H + NW - 1) / NW;
    const uint64_t nblk = (uint64_t)yblocks * tiles_x * nz;
    const Field fp{"p", true}, fpp{"pp", false}, fc2{"c2", false}, fpeer{"peer plane", false};
    std::vector<unsigned char> seen((size_t)nz * H * pitch / 4 + 1, 0);
    for (uint64_t blk = 0; blk < nblk; ++blk) {
        const RowCoord rc = row_coord(blk, yblocks, tiles_x, nz, slab);
        const uint32_t x0 = rc.tx * 128u, y0 = rc.yb * (uint32_t)NW;
        for (int w = 0; w < NW; ++w)
            for (int lane = 0; lane < 32; ++lane) {
                const uint32_t x = x0 + 4u * (uint32_t)lane, y = y0 + (uint32_t)w;
                const bool xin = x < pitch, act = xin && y < H;
                const int64_t o = (int64_t)rc.z * P + (int64_t)y * pitch + x;
                if (act) {
                    seen[(((size_t)rc.z * H + y) * pitch + x) / 4]++;
                    check(fp, o, 4, pitch, nz, P, "rows centre", rc.tx, y, rc.z, lane, w);
                    check(fp, o - P, 4, pitch, nz, P, "rows z-1", rc.tx, y, rc.z, lane, w);
                    check(fp, o + P, 4, pitch, nz, P, "rows z+1", rc.tx, y, rc.z, lane, w);
                    check(fpp, o, 4, pitch, nz, P, "rows p_prev / store", rc.tx, y, rc.z, lane, w);
                    check(fc2, o, 4, pitch, nz, P, "rows c2", rc.tx, y, rc.z, lane, w);
                    if (lane == 0 && x0 > 0)
                        check(fp, o - 1, 1, pitch, nz, P, "rows x-1", rc.tx, y, rc.z, lane, w);
                    if (lane == 31 && x0 + 128u < pitch)
                        check(fp, o + 4, 1, pitch, nz, P, "rows x+128", rc.tx, y, rc.z, lane, w);
                    if (slab && (rc.z == 0 || rc.z + 1 == nz))
                        check(fpeer, (int64_t)y * pitch + x, 4, pitch, 1, P, "rows peer store",
                              rc.tx, y, rc.z, lane, w);
                }
                if (xin && w == 0)
                    check(fp, (int64_t)rc.z * P + ((int64_t)y0 - 1) * pitch + x, 4, pitch, nz, P,
                          "rows halo y0-1", rc.tx, y, rc.z, lane, w);
                if (xin && w == NW - 1 && y0 + NW <= H)
                    check(fp, (int64_t)rc.z * P + ((int64_t)y0 + NW) * pitch + x, 4, pitch, nz, P,
                          "rows halo y0+NW", rc.tx, y, rc.z, lane, w);
            }
    }
    for (uint32_t z = 0; z < nz; ++z)
        for (uint32_t y = 0; y < H; ++y)
            for (uint32_t x = 0; x < pitch; x += 4) {
                const size_t c = (((size_t)z * H + y) * pitch + x) / 4;
                if (seen[c] != 1) {
                    if (g_bad < 20)
                        fprintf(stderr, "rows: float4 at (%u,%u,%u) covered %d times\n", x, y, z,
                                seen[c]);
                    ++g_bad;
                }
            }
}

// k_persistent_smem: the block shape the host picks (smem_step_shape, 148
// SMs, 220 KiB, with or without a c2 field), then every shared-memory index the kernel forms (loads, the
// cell rule's six neighbours, sources anywhere in the block and its halo,
// faces, halo rows, the final write) against the two volumes and the c2
// block, and every global offset against the owned planes; every cell of
// the grid owned by exactly one block.
static void run_smem(uint32_t W, uint32_t H, uint32_t nz, bool c2f) {
    const uint32_t pitch = (W + 31u) & ~31u;
    const int64_t P = (int64_t)H * pitch;
    uint32_t by = 0, bz = 0;
    if (!smem_step_shape(pitch, H, nz, 148, c2f, 220u * 1024u, &by, &bz)) {
        printf("no shared-memory shape for %u x %u x %u (the row body takes it)\n", W, H, nz);
        return;
    }
    const int SX = (int)pitch + 2, SY = (int)by + 2, SP = SX * SY, SV = SP * ((int)bz + 2);
    const uint64_t c2n = (uint64_t)pitch * by * bz;
    if (smem_step_bytes(pitch, by, bz, c2f) != (uint64_t)(2 * SV) * 4 + (c2f ? c2n * 4 : 0)) ++g_bad;
    const uint32_t yblocks = (H + by - 1) / by, zblocks = (nz + bz - 1) / bz;
    std::vector<unsigned char> owner((size_t)nz * H, 0);
    // exchange rows: [block][slot] -> global rows (z * H + y) stored there
    std::vector<std::vector<int64_t>> sent((size_t)yblocks * zblocks * smem_xch_rows(by, bz));
    auto sm_ok = [&](int x, int y, int z, const char* what) {
        ++g_checked;
        const int64_t i = (int64_t)(z + 1) * SP + (int64_t)(y + 1) * SX + (x + 1);
        if (x < -1 || x > (int)pitch || i < 0 || i >= SV) {
            if (g_bad < 20) fprintf(stderr, "SMEM OUT OF BOUNDS %s (%d,%d,%d) i=%lld\n", what, x, y, z,
                                    (long long)i);
            ++g_bad;
        }
    };
    auto g_ok = [&](uint32_t x, int64_t y, int64_t z, const char* what) {
        ++g_checked;
        if (x >= pitch || y < 0 || y >= (int64_t)H || z < 0 || z >= (int64_t)nz) {
            if (g_bad < 20) fprintf(stderr, "GLOBAL OUT OF RANGE %s (%u,%lld,%lld)\n", what, x,
                                    (long long)y, (long long)z);
            ++g_bad;
        }
        (void)P;
    };
    for (uint32_t blk = 0; blk < yblocks * zblocks; ++blk) {
        const uint32_t y0 = (blk % yblocks) * by, z0 = (blk / yblocks) * bz;
        const uint32_t ny = by < H - y0 ? by : H - y0, nzb = bz < nz - z0 ? bz : nz - z0;
        for (int zz = -1; zz <= (int)nzb; ++zz)   // loads (in-grid rows only) and sources
            for (int yy = -1; yy <= (int)ny; ++yy)
                for (uint32_t x = 0; x < pitch; ++x) {
                    sm_ok((int)x, yy, zz, "load / source");
                    const int64_t gz = (int64_t)z0 + zz, gy = (int64_t)y0 + yy;
                    if (gz >= 0 && gz < (int64_t)nz && gy >= 0 && gy < (int64_t)H)
                        g_ok(x, gy, gz, "load");
                }
        for (int zz = 0; zz < (int)nzb; ++zz)
            for (int yy = 0; yy < (int)ny; ++yy) {
                owner[(size_t)(z0 + zz) * H + y0 + yy]++;
                for (uint32_t x = 0; x < pitch; ++x) {
                    sm_ok((int)x - 1, yy, zz, "w");
                    sm_ok((int)x + 1, yy, zz, "e");
                    sm_ok((int)x, yy - 1, zz, "s");
                    sm_ok((int)x, yy + 1, zz, "n");
                    sm_ok((int)x, yy, zz - 1, "d");
                    sm_ok((int)x, yy, zz + 1, "u");
                    ++g_checked;
                    if ((uint64_t)(((uint64_t)zz * by + yy) * pitch + x) >= c2n) ++g_bad;
                    g_ok(x, (int64_t)y0 + yy, (int64_t)z0 + zz, "face / final write");
                }
            }
        // face rows into the neighbours' exchange rows (smem_face_dest)
        const uint32_t yb = blk % yblocks, zb = blk / yblocks;
        for (int r = 0; r < 2 * (int)nzb + 2 * (int)ny; ++r) {
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
            uint32_t nb;
            int side, i;
            ++g_checked;
            if (!smem_face_dest(blk, yblocks, zblocks, kind, yy, zz, &nb, &side, &i)) {
                const bool edge = kind == 0 ? yb == 0 : kind == 1 ? yb + 1 == yblocks
                                : kind == 2 ? zb == 0 : zb + 1 == zblocks;
                if (!edge) ++g_bad;   // a neighbour exists but gets nothing
                continue;
            }
            const uint32_t slot = smem_xch_slot(by, bz, side, i);
            if (nb >= yblocks * zblocks || slot >= smem_xch_rows(by, bz)) {
                if (g_bad < 20) fprintf(stderr, "smem xch: block %u row (%d,%d) -> %u slot %u\n",
                                        blk, yy, zz, nb, slot);
                ++g_bad;
                continue;
            }
            sent[(size_t)nb * smem_xch_rows(by, bz) + slot].push_back(
                (int64_t)(z0 + zz) * H + (y0 + yy));
        }
    }
    // every in-grid halo row a block reads comes from exactly one face row,
    // the same global row; the halo rows stay inside the shared volume
    for (uint32_t blk = 0; blk < yblocks * zblocks; ++blk) {
        const uint32_t yb = blk % yblocks, zb = blk / yblocks;
        const uint32_t y0 = yb * by, z0 = zb * bz;
        const uint32_t ny = by < H - y0 ? by : H - y0, nzb = bz < nz - z0 ? bz : nz - z0;
        std::vector<unsigned char> used(smem_xch_rows(by, bz), 0);
        for (int r = 0; r < 2 * (int)nzb + 2 * (int)ny; ++r) {
            int yy, zz, side, i;
            bool have;
            if (r < 2 * (int)nzb) {
                zz = r >> 1;
                side = r & 1;
                yy = side ? (int)ny : -1;
                i = zz;
                have = side ? yb + 1 < yblocks : yb > 0;
            } else {
                yy = (r - 2 * (int)nzb) >> 1;
                side = 2 + ((r - 2 * (int)nzb) & 1);
                zz = side == 3 ? (int)nzb : -1;
                i = yy;
                have = side == 3 ? zb + 1 < zblocks : zb > 0;
            }
            const int64_t gy = (int64_t)y0 + yy, gz = (int64_t)z0 + zz;
            const bool in_grid = gy >= 0 && gy < (int64_t)H && gz >= 0 && gz < (int64_t)nz;
            ++g_checked;
            if (have != in_grid) ++g_bad;   // a halo row in the grid must have a sender
            if (!have) continue;
            for (uint32_t x = 0; x < pitch; ++x) sm_ok((int)x, yy, zz, "halo");
            const uint32_t slot = smem_xch_slot(by, bz, side, i);
            ++g_checked;
            if (slot >= used.size() || used[slot]++) {
                ++g_bad;
                continue;
            }
            const auto& got = sent[(size_t)blk * smem_xch_rows(by, bz) + slot];
            ++g_checked;
            if (got.size() != 1 || got[0] != gz * (int64_t)H + gy) {
                if (g_bad < 20) fprintf(stderr, "smem xch: block %u halo (%d,%d) slot %u gets %zu rows\n",
                                        blk, yy, zz, slot, got.size());
                ++g_bad;
            }
        }
    }
    for (size_t r = 0; r < owner.size(); ++r)
        if (owner[r] != 1) {
            if (g_bad < 20) fprintf(stderr, "smem: row %zu owned %d times\n", r, owner[r]);
            ++g_bad;
        }
    printf("shape %u x %u x %u, %u blocks\n", pitch, by, bz, yblocks * zblocks);
}

int main(int argc, char** argv) {
    if (argc < 5) {
        fprintf(stderr, "usage: %s W H nz sm_count [TY]\n", argv[0]);
        return 2;
    }
    const uint32_t W = (uint32_t)atoi(argv[1]), H = (uint32_t)atoi(argv[2]),
                   nz = (uint32_t)atoi(argv[3]);
    const int sms = atoi(argv[4]);
    const int ty = argc > 5 ? atoi(argv[5]) : 8;
    const bool halo = argc > 6 && atoi(argv[6]) != 0;
    if (argc > 7 && atoi(argv[7]) == 3) {
        run_smem(W, H, nz, halo);   // the sixth argument selects a c2 field here
        printf("checked %lld accesses, %d out of bounds\n", g_checked, g_bad);
        return g_bad == 0 ? 0 : 1;
    }
    if (argc > 7 && atoi(argv[7]) == 2) {
        run_rows(W, H, nz, halo, ty);
        printf("checked %lld accesses, %d out of bounds\n", g_checked, g_bad);
        return g_bad == 0 ? 0 : 1;
    }
    if (argc > 7 && atoi(argv[7]) == 1) {
        run_async(W, H, nz, sms, halo);
        printf("checked %lld accesses, %d out of bounds\n", g_checked, g_bad);
        return g_bad == 0 ? 0 : 1;
    }
    switch (ty) {
        case 4: run<4>(W, H, nz, sms, halo); break;
        case 8: run<8>(W, H, nz, sms, halo); break;
        case 16: run<16>(W, H, nz, sms, halo); break;
        default: fprintf(stderr, "TY must be 4, 8 or 16\n"); return 2;
    }
    printf("checked %lld accesses, %d out of bounds\n", g_checked, g_bad);
    return g_bad == 0 ? 0 : 1;
}
