// Accuracy of kd::exp2_poly (the FMA-pipe exp2 used for part of the softmax) on the GPU:
// evaluates it on a dense grid over the argument range the softmax produces ([-130, 8],
// plus -inf) and compares with exp2 in double on the host; and checks that the packed
// kd::exp2_poly2 returns exactly exp2_poly's bits for every pair of grid points.  Prints
// "max_rel <value> zero_ok <0|1> pair_equal <0|1>".  Built and run by tests/test_gpu_exp2.py.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "kd_common.cuh"

__global__ void eval(const float* x, float* y, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = kd::exp2_poly(x[i]);
}

__global__ void eval2(const float* x, float* y, int n) {  // pairs (x[i], x[n-1-i])
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) kd::exp2_poly2(x[i], x[n - 1 - i], y[2 * i], y[2 * i + 1]);
}

int main() {
    const int n = 1 << 22;
    std::vector<float> hx(n), hy(n);
    for (int i = 0; i < n - 1; ++i) hx[i] = -130.0f + 138.0f * (float)i / (float)(n - 2);
    hx[n - 1] = -INFINITY;
    float *dx = nullptr, *dy = nullptr;
    if (cudaMalloc(&dx, n * 4) != cudaSuccess || cudaMalloc(&dy, n * 4) != cudaSuccess) return 2;
    cudaMemcpy(dx, hx.data(), n * 4, cudaMemcpyHostToDevice);
    eval<<<(n + 255) / 256, 256>>>(dx, dy, n);
    if (cudaMemcpy(hy.data(), dy, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return 3;
    double worst = 0.0;
    int zero_ok = 1;
    for (int i = 0; i < n; ++i) {
        const double x = hx[i];
        if (!(x > -126.0)) {  // documented: exactly 0 at or below -126 (and for -inf)
            if (hy[i] != 0.0f) zero_ok = 0;
            continue;
        }
        const double ref = std::exp2(x);
        if (ref < 1.5e-38) continue;  // results in the subnormal range carry absolute, not relative, error
        const double rel = std::fabs((double)hy[i] - ref) / ref;
        if (rel > worst) worst = rel;
    }
    float* dy2 = nullptr;
    std::vector<float> hy2(2 * (size_t)n);
    if (cudaMalloc(&dy2, 2 * (size_t)n * 4) != cudaSuccess) return 2;
    eval2<<<(n + 255) / 256, 256>>>(dx, dy2, n);
    if (cudaMemcpy(hy2.data(), dy2, 2 * (size_t)n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return 3;
    int pair_equal = 1;
    for (int i = 0; i < n; ++i) {
        uint32_t a, b, c, d;
        memcpy(&a, &hy2[2 * i], 4);
        memcpy(&b, &hy[i], 4);
        memcpy(&c, &hy2[2 * i + 1], 4);
        memcpy(&d, &hy[n - 1 - i], 4);
        if (a != b || c != d) pair_equal = 0;
    }
    cudaFree(dy2);
    printf("max_rel %.6e zero_ok %d pair_equal %d\n", worst, zero_ok, pair_equal);
    cudaFree(dx);
    cudaFree(dy);
    return 0;
}
