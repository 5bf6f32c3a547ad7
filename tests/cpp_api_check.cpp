// C++ API check (run by tests/test_cpp_api.py on a GPU): the header-only
// mirror of GpuBackend3D / PersistentBackend (include/ws3d.hpp) against the
// CPU oracle's C restatement, linked directly.  Prints "CPP-API OK".
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include "ws3d.hpp"

extern "C" {
typedef struct {
    float c_squared, damping;
    const float* c2_field;
    const float* sponge;
    uint32_t sponge_w;
} ws3o_params;
void ws3o_run(uint32_t, uint32_t, uint32_t, float*, float*, const uint8_t*, const float*,
              const ws3o_params*, uint64_t, uint64_t, uint32_t, const uint64_t*, const float*,
              uint64_t, int);
void ws3o_inject_impulse(uint32_t, uint32_t, uint32_t, float*, float*, uint32_t, uint32_t,
                         uint32_t, float);
}

int main() {
    const uint32_t W = 150, H = 40, D = 36;
    const size_t N = (size_t)W * H * D;
    std::vector<float> p(N, 0.0f), pp(N, 0.0f);
    for (size_t i = 0; i < N; ++i) p[i] = pp[i] = (float)std::sin(0.001 * (double)i);
    ws3d::GridDims g{W, H, D};
    g.damping = 0.9995f;

    // oracle: impulse, 40 steps
    std::vector<float> rp = p, rpp = pp;
    ws3o_inject_impulse(W, H, D, rp.data(), rpp.data(), 70, 20, 18, 1.0f);
    ws3o_params prm{0.25f, 0.9995f, nullptr, nullptr, 0};
    ws3o_run(W, H, D, rp.data(), rpp.data(), nullptr, nullptr, &prm, 0, 40, 0, nullptr, nullptr,
             0, 1);

    int bad = 0;
    for (int mode = 0; mode < 2; ++mode) {
        std::vector<float> out(N);
        if (mode == 0) {
            ws3d::GpuBackend3D gpu(g, p.data(), pp.data());
            gpu.inject_impulse(70, 20, 18, 1.0f);
            for (int s = 0; s < 40; ++s) gpu.step();
            gpu.download_pressure(out.data());
            if (gpu.memory_usage() < 2 * N * sizeof(float)) ++bad;
        } else {
            ws3d::PersistentBackend pb(g, p.data(), pp.data());
            pb.inject_impulse(70, 20, 18, 1.0f);
            pb.step(40);
            pb.download_pressure(out.data());
        }
        if (std::memcmp(out.data(), rp.data(), N * sizeof(float)) != 0) {
            std::printf("mode %d differs from the oracle\n", mode);
            ++bad;
        }
    }
    // errors surface as exceptions, never as a silent fallback
    try {
        ws3d::GridDims z{0, 4, 4};
        ws3d::GpuBackend3D broken(z);
        ++bad;
    } catch (const ws3d::GpuError& e) {
        if (e.status != WS3D_EINVAL) ++bad;
    }
    std::printf(bad ? "CPP-API FAIL\n" : "CPP-API OK\n");
    return bad ? 1 : 0;
}
