// Test kernel: the largest relative difference between the kernels' branch-free double exp
// (lrs::exp_neg) and CUDA's double exp over every float d in [-104, 0), and the number of
// those d where the two, rounded to float, differ while CUDA's double exp lies farther than
// 2^-20 float ulp from the rounding midpoint (the margin the kernels' midpoint test keeps).
// out[0]: the maximum relative difference (float bits); out[1]: that count.
#include <cuda_runtime.h>
#include <cstdint>

#include "../../llama.rs_b200/csrc/lrs_device.cuh"

__global__ void exp_neg_diff(unsigned* out) {
    const uint32_t lo = 0x80000001u, hi = 0xC2D00000u;  // -tiny .. -104
    const uint64_t span = (uint64_t)(hi - lo) + 1u;
    float m = 0.0f;
    unsigned bad = 0;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < span;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const float d = __uint_as_float(lo + (uint32_t)i);
        const double ref = exp((double)d), mine = lrs::exp_neg((double)d);
        m = fmaxf(m, (float)(fabs(mine - ref) / ref));
        const float er = __double2float_rn(ref), em = __double2float_rn(mine);
        if (er != em && er >= 1.1754943508222875e-38f) {
            const uint32_t eb = __float_as_uint(er);
            const double ec = (double)er, nb = (double)__uint_as_float(ref >= ec ? eb + 1u : eb - 1u);
            if (fabs(ref - ec) < (0.5 - 0x1p-20) * fabs(nb - ec)) ++bad;
        }
    }
    atomicMax(out, __float_as_uint(m));
    if (bad) atomicAdd(out + 1, bad);
}

extern "C" int lrs_test_exp_neg(unsigned* host_out) {
    unsigned* d_out = nullptr;
    if (cudaMalloc(&d_out, 2 * sizeof(unsigned)) != cudaSuccess) return 1;
    cudaMemset(d_out, 0, 2 * sizeof(unsigned));
    exp_neg_diff<<<148 * 8, 256>>>(d_out);
    int rc = (int)cudaDeviceSynchronize();
    if (rc == 0) rc = (int)cudaMemcpy(host_out, d_out, 2 * sizeof(unsigned), cudaMemcpyDeviceToHost);
    cudaFree(d_out);
    return rc;
}
