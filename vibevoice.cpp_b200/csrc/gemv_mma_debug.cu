// gemv_mma_debug.cu -- test hook for the tensor-core decode GEMV math of
// gemv_mma.cuh: one CTA quantizes M <= 2 activation rows into their pieces,
// then each warp multiplies 16-row groups of a device Q8_0 matrix (read from
// global memory) and writes y[m][row].  Checked against the CPU oracle's exact
// matvec by the GPU tests; the persistent decode step uses the same routines.
#include "common.cuh"
#include "gemv_mma.cuh"
#include "kernels.h"

namespace vvq2 {

namespace {

constexpr int DG_THREADS = 512;

template <int MB>
__global__ void __launch_bounds__(DG_THREADS) k_debug_gemv_mma(const DevW w, const float* x, float* y) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int K = w.cols, N = w.rows, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const gm::ActQ aq = gm::actq_at(sm, MB, K);
    float* red = reinterpret_cast<float*>(sm + ((gm::actq_bytes(MB, K) + 15) / 16) * 16);   // [16 warps][16][8]
    const int K4 = K / 4;
    // every lane of a warp takes part (the block reductions are warp shuffles)
    for (int i0 = 0; i0 < MB * K4; i0 += DG_THREADS) {
        const int i = i0 + tid;
        const bool valid = i < MB * K4;
        const int m = valid ? i / K4 : 0, k4 = valid ? i % K4 : 0;
        const float4 v = valid ? reinterpret_cast<const float4*>(x + (size_t)m * K)[k4] : make_float4(0, 0, 0, 0);
        gm::quantize_group(aq, m, k4, v, valid);
    }
    __syncthreads();
    float* r = red + warp * 16 * 8;
    for (int row0 = 16 * warp; row0 < N; row0 += 16 * (DG_THREADS / 32)) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        gm::tile_mma<MB>(w.q, (int)w.row_stride, K, row0, min(16, N - row0), 0, K / 32, aq, lane,
                         acc);
        // this tile's rows start at row0: tile_mma indexes rows row0 + g from w.q
        const int g = lane >> 2, t = lane & 3;
        r[g * 8 + 2 * t] = acc[0];
        r[g * 8 + 2 * t + 1] = acc[1];
        r[(g + 8) * 8 + 2 * t] = acc[2];
        r[(g + 8) * 8 + 2 * t + 1] = acc[3];
        __syncwarp();
        if (lane < 16 * MB) {
            const int rr = lane % 16, m = lane / 16;
            if (row0 + rr < N)
                y[(size_t)m * N + row0 + rr] = r[rr * 8 + 3 * m] + r[rr * 8 + 3 * m + 1] + r[rr * 8 + 3 * m + 2];
        }
        __syncwarp();
    }
}

}  // namespace

cudaError_t debug_gemv_mma_launch(const DevW& w, const float* x, int M, float* y, cudaStream_t st) {
    if (M < 1 || M > 2 || w.type != W_Q8_0 || w.cols % 32) return cudaErrorInvalidValue;
    const size_t smem = ((gm::actq_bytes(M, w.cols) + 15) / 16) * 16 + 16 * 16 * 8 * sizeof(float);
    cudaError_t e;
    if (M == 1) {
        e = cudaFuncSetAttribute(k_debug_gemv_mma<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_debug_gemv_mma<1><<<1, DG_THREADS, smem, st>>>(w, x, y);
    } else {
        e = cudaFuncSetAttribute(k_debug_gemv_mma<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_debug_gemv_mma<2><<<1, DG_THREADS, smem, st>>>(w, x, y);
    }
    note_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace vvq2
