// Test kernel: the largest relative error of CUDA's expf(d) against the double-precision
// exp(d), per unit interval of d in [-104, 0), over every float d whose exact result is a
// normal float.  The sampling kernels classify an element by CUDA's expf and take libm's
// value wherever the two could round differently; that test assumes a relative error
// below 2^-21, which this measures.  out[b] (b = floor(-d), 0..103): float bits of the
// maximum (non-negative float bits order as the floats do, so atomicMax takes it).
#include <cuda_runtime.h>
#include <cstdint>

__global__ void expf_error(unsigned* out) {
    const uint32_t lo = 0x80000001u, hi = 0xC2D00000u;  // -tiny .. -104
    const uint64_t span = (uint64_t)(hi - lo) + 1u;
    int cb = -1;
    float m = 0.0f;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < span;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const float d = __uint_as_float(lo + (uint32_t)i);
        const double ex = exp((double)d);
        if (ex < 1.1754943508222875e-38) continue;  // (subnormal results: the kernels take libm's)
        int b = (int)(-d);
        if (b > 103) b = 103;
        if (b != cb) {
            if (cb >= 0) atomicMax(out + cb, __float_as_uint(m));
            cb = b;
            m = 0.0f;
        }
        m = fmaxf(m, (float)(fabs((double)expf(d) - ex) / ex));
    }
    if (cb >= 0) atomicMax(out + cb, __float_as_uint(m));
}

extern "C" int lrs_test_expf_error(unsigned* host_out) {
    unsigned* d_out = nullptr;
    if (cudaMalloc(&d_out, 104 * sizeof(unsigned)) != cudaSuccess) return 1;
    cudaMemset(d_out, 0, 104 * sizeof(unsigned));
    expf_error<<<148 * 8, 256>>>(d_out);
    int rc = (int)cudaDeviceSynchronize();
    if (rc == 0) rc = (int)cudaMemcpy(host_out, d_out, 104 * sizeof(unsigned), cudaMemcpyDeviceToHost);
    cudaFree(d_out);
    return rc;
}
