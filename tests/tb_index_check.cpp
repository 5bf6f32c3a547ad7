// Host-side bounds check of the two-step kernel's explicit global accesses on
// one GPU and on z-slabs (rustcompute_b200/csrc/ws3d_tb.cuh, k_step_tma2).
//
// TMA box loads are clipped by the hardware; what the kernel addresses itself
// is replayed here for every item of the launch schedule (tb_schedule, the
// same helper the host uses), every consumer warp and lane:
//   - float4 stores of X(q) and Y(q-1) into the context's own buffers
//     (planes [zs, ze) of the run, rows y < H, x < pitch);
//   - slabs: Y of planes 0, 1 / nz-2, nz-1 stored into the neighbours' Y
//     buffers (their ghost planes nz_lo, nz_lo+1 / -1, -2);
//   - slabs: the plane coordinates of the producer's TMA boxes of the
//     neighbours' own edge planes (p_{t-1} and c2);
//   - the single-step kernel's two-plane stores into the neighbours at
//     temporal depth 2 and the source-ghost offsets of the host.
// Allocations: a slab's field buffer holds planes [-2, nz + 2), the c2 field
// [-1, nz + 1); one GPU's buffers [-1, nz + 1).  Every access must lie inside
// its allocation, be 16-byte aligned for float4 and stay inside one row.
// Usage: tb_index_check W H nz lo_nz hi_nz [sm_count]   (0 = no neighbour)
#include <cstdio>
#include <cstdlib>

#include "ws3d_index.h"

using namespace ws3d;

static long long g_checked = 0;
static int g_bad = 0;

// offset o (floats, relative to plane 0 of a buffer with planes [plo, phi))
static void check(const char* what, int64_t o, int n, int64_t plane, uint32_t pitch, int plo,
                  int phi, int item, int w, int lane) {
    ++g_checked;
    const int64_t lo = (int64_t)plo * plane, hi = (int64_t)phi * plane;
    const int64_t in_row = ((o % (int64_t)pitch) + pitch) % (int64_t)pitch;
    bool ok = o >= lo && o + n <= hi && in_row + n <= (int64_t)pitch;
    if (n == 4 && (o % 4) != 0) ok = false;
    if (!ok && g_bad < 20)
        fprintf(stderr, "OUT OF BOUNDS %s off=%lld n=%d [%lld,%lld) item=%d w=%d lane=%d\n", what,
                (long long)o, n, (long long)lo, (long long)hi, item, w, lane);
    if (!ok) ++g_bad;
}

int main(int argc, char** argv) {
    if (argc < 6) {
        fprintf(stderr, "usage: tb_index_check W H nz lo_nz hi_nz [sm_count]\n");
        return 2;
    }
    const uint32_t W = (uint32_t)atoi(argv[1]), H = (uint32_t)atoi(argv[2]);
    const uint32_t nz = (uint32_t)atoi(argv[3]);
    const uint32_t lo_nz = (uint32_t)atoi(argv[4]), hi_nz = (uint32_t)atoi(argv[5]);
    const int sms = argc > 6 ? atoi(argv[6]) : 148;
    const bool has_lo = lo_nz > 0, has_hi = hi_nz > 0;
    const bool slab = has_lo || has_hi;
    const int gd = slab ? 2 : 1;
    constexpr int TY = kTbTY;
    const uint32_t pitch = (W + 31u) & ~31u;
    const int64_t P = (int64_t)H * pitch;
    const uint32_t tiles_x = (pitch + 127) / 128;
    const uint32_t tiles = tiles_x * ((H + TY - 1) / TY);
    const TmaSchedule sch = tb_schedule(tiles, nz, (uint32_t)(kTbCtasPerSm * sms));
    for (uint32_t item = 0; item < sch.nitems; ++item) {
        const uint32_t chunk = item / tiles, tile = item - chunk * tiles;
        const int zs = (int)(chunk * sch.clen);
        const int ze = (int)(nz < chunk * sch.clen + sch.clen ? nz : chunk * sch.clen + sch.clen);
        const uint32_t x0 = (tile % tiles_x) * 128u, y0 = (tile / tiles_x) * TY;
        const bool push_lo = has_lo && zs < 2, push_hi = has_hi && ze + 2 > (int)nz;
        for (int w = 0; w < TY + 2; ++w) {
            const bool do_y = w >= 1 && w <= TY;
            for (int lane = 0; lane < 32; ++lane) {
                const uint32_t x = x0 + 4u * lane;
                const uint32_t y = y0 + (uint32_t)w - 1u;
                const bool act = do_y && x < pitch && y < H;
                const int64_t row = (int64_t)y * pitch + x;
                // X(q) for q in [zs, ze): the item loop runs q = zs-1 .. ze
                for (int q = zs - 1; q <= ze; ++q) {
                    if (act && q >= zs && q < ze)
                        check("X store", (int64_t)q * P + row, 4, P, pitch, -gd, (int)nz + gd,
                              (int)item, w, lane);
                    const int qy = q - 1;
                    if (!(do_y && qy >= zs && qy < ze) || !act) continue;
                    check("Y store", (int64_t)qy * P + row, 4, P, pitch, -gd, (int)nz + gd,
                          (int)item, w, lane);
                    if (push_lo && qy < 2)   // lower neighbour: its planes lo_nz + qy
                        check("Y push lo", (int64_t)(lo_nz + qy) * P + row, 4, P, pitch, -2,
                              (int)lo_nz + 2, (int)item, w, lane);
                    if (push_hi && qy + 2 >= (int)nz)   // upper: its planes qy - nz (-1, -2)
                        check("Y push hi", ((int64_t)qy - (int64_t)nz) * P + row, 4, P, pitch, -2,
                              (int)hi_nz + 2, (int)item, w, lane);
                }
            }
        }
        // the producer's TMA boxes of p_{t-1} and c2 for the ghost planes -1 / nz
        // come from the neighbour's own buffers (maps over its planes -1 .. nz_nb,
        // coordinate = plane + 1): its last plane / its plane 0, whole boxes
        // inside the map's plane range (x and y are clipped by the hardware)
        for (int i = 2; i <= (ze - zs) + 3; ++i) {
            const int q = zs - 3 + i;
            ++g_checked;
            if (q < 0 && has_lo) {
                const int zc = (int)lo_nz;   // its plane lo_nz - 1
                if (!(zc >= 0 && zc < (int)lo_nz + 2)) {
                    if (g_bad < 20) fprintf(stderr, "OUT OF BOUNDS peer B/c2 lo plane %d\n", zc);
                    ++g_bad;
                }
            } else if (q >= (int)nz && has_hi) {
                const int zc = 1;            // its plane 0
                if (!(zc >= 0 && zc < (int)hi_nz + 2)) {
                    if (g_bad < 20) fprintf(stderr, "OUT OF BOUNDS peer B/c2 hi plane %d\n", zc);
                    ++g_bad;
                }
            } else if (q < -1 || q > (int)nz) {
                if (g_bad < 20) fprintf(stderr, "own B/c2 box outside planes -1..nz: %d\n", q);
                ++g_bad;
            }
        }
    }
    // single-step kernel at depth 2: planes 0, 1 / nz-1, nz-2 into the neighbours
    for (uint32_t y = 0; y < H; ++y)
        for (uint32_t x = 0; x < pitch; x += 4) {
            const int64_t row = (int64_t)y * pitch + x;
            for (uint32_t z = 0; z < nz; ++z) {
                if (has_lo && z == 0) check("tma push lo", (int64_t)lo_nz * P + row, 4, P, pitch,
                                            -2, (int)lo_nz + 2, -1, -1, -1);
                if (has_lo && z == 1) check("tma push lo2", (int64_t)(lo_nz + 1) * P + row, 4, P,
                                            pitch, -2, (int)lo_nz + 2, -1, -1, -1);
                if (has_hi && z + 1 == nz) check("tma push hi", -P + row, 4, P, pitch, -2,
                                                 (int)hi_nz + 2, -1, -1, -1);
                if (has_hi && z + 2 == nz) check("tma push hi2", -2 * P + row, 4, P, pitch, -2,
                                                 (int)hi_nz + 2, -1, -1, -1);
            }
            // source ghosts: lower relative to its plane -1 (+ lo_nz + 1 planes to its upper
            // ghost), upper relative to its plane -2; depth 2 for sources on the edge planes
            for (uint32_t from = 0; from < 2 && from < nz; ++from) {
                if (has_lo) check("src ghost lo", -P + (int64_t)(lo_nz + 1) * P + (int64_t)from * P +
                                                      row, 1, P, pitch, -2, (int)lo_nz + 2,
                                  -1, -1, -1);
                if (has_hi) check("src ghost hi", -2 * P + (1 - (int64_t)from) * P + row, 1, P,
                                  pitch, -2, (int)hi_nz + 2, -1, -1, -1);
            }
        }
    printf("checked %lld accesses, %d out of bounds (clen %u, %u items)\n", g_checked, g_bad,
           sch.clen, sch.nitems);
    return g_bad ? 1 : 0;
}
