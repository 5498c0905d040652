// The reference C test's 5-point FFT (tests/test_c_api.c:49-108) through the
// C++ owners of include/cubutterfly/plan.hpp: Context, Plan with an owned
// workspace, execute, inverse round trip.
#include <cubutterfly/plan.hpp>

#include <cmath>
#include <cstdio>
#include <vector>

int main() {
    cubutterfly::Context context;
    cudaStream_t stream = nullptr;
    if (cudaStreamCreate(&stream) != cudaSuccess) return 2;
    context.set_stream(stream);
    cubutterfly::Transform t;
    t.extents = {5};
    cubutterfly::Plan forward(context, t);
    t.inverse = true;
    cubutterfly::Plan inverse(context, t);
    std::vector<float> x(10, 0.f), y(10), z(10);
    x[2] = 1.f;  // impulse at index 1 (interleaved complex)
    void *dx = nullptr, *dy = nullptr, *dz = nullptr;
    cudaMalloc(&dx, 80);
    cudaMalloc(&dy, 80);
    cudaMalloc(&dz, 80);
    cudaMemcpyAsync(dx, x.data(), 40, cudaMemcpyHostToDevice, stream);
    forward.execute(dx, dy);
    inverse.execute_steady(dy, dz);
    cudaMemcpyAsync(y.data(), dy, 40, cudaMemcpyDeviceToHost, stream);
    cudaMemcpyAsync(z.data(), dz, 40, cudaMemcpyDeviceToHost, stream);
    cudaStreamSynchronize(stream);
    int bad = 0;
    for (int k = 0; k < 5; ++k) {
        const double a = -2.0 * 3.14159265358979323846 * k / 5.0;
        bad += std::fabs(y[2 * k] - std::cos(a)) > 2e-5 || std::fabs(y[2 * k + 1] - std::sin(a)) > 2e-5;
        bad += std::fabs(z[2 * k] - x[2 * k]) > 2e-5 || std::fabs(z[2 * k + 1] - x[2 * k + 1]) > 2e-5;
    }
    std::printf("%s %s %zu\n", bad ? "failed" : "ok", forward.algorithm_name().c_str(), forward.workspace_size());
    cudaFree(dx);
    cudaFree(dy);
    cudaFree(dz);
    cudaStreamDestroy(stream);
    return bad;
}
