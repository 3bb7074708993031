// Accuracy of kd::exp2_poly (the FMA-pipe exp2 used for part of the softmax) on the GPU:
// evaluates it on a dense grid over the argument range the softmax produces ([-130, 8],
// plus -inf) and compares with exp2 in double on the host.  Prints
// "max_rel <value> zero_ok <0|1>".  Built and run by tests/test_gpu_exp2.py.
#include <cmath>
#include <cstdio>
#include <vector>

#include "kd_common.cuh"

__global__ void eval(const float* x, float* y, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = kd::exp2_poly(x[i]);
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
    printf("max_rel %.6e zero_ok %d\n", worst, zero_ok);
    cudaFree(dx);
    cudaFree(dy);
    return 0;
}
