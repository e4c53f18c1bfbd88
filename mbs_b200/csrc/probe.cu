// Tensor-pipe peak probe for tcgen05.mma kind::mxf4 (diagnostic entry point).
//
// The roofline denominator of a compute-bound MXFP4 GEMM: every CTA pair of
// the GPU issues back-to-back 256 x 256 x 64 pair MMAs (the prefill kernel's
// instruction) on operands that stay resident in shared memory, with block
// scales resident in TMEM, so nothing but the tensor pipe limits the rate.
// Reported: TFLOP/s over the whole grid (CUDA events), cycles per MMA and the
// SM clock seen (clock64 / %globaltimer on each leader CTA).
#include "common.h"
#include "ptx.cuh"

namespace mbs {
namespace probe {
namespace {

constexpr int kThreads = 128;
constexpr int kSmem = 120 * 1024;  // forces one CTA per SM
constexpr int kMmaPerGroup = 4;    // one 256-element K stage
constexpr int kMaxCtas = 1024;

__device__ unsigned long long g_cycles[kMaxCtas];
__device__ unsigned long long g_ns[kMaxCtas];

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    mxf4_peak_probe_kernel(int groups, unsigned* err)
{
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint64_t bar_loop, bar_end;
    __shared__ uint32_t tslot;
    uint8_t* a = smem;             // 128 rows x 128 B, 128-byte swizzled K-major
    uint8_t* b = smem + 16384;     // this CTA's 128-row half of B, no-swizzle K-major
    uint8_t* sf = smem + 32768;    // 6 scale blocks of 32 x 16 B
    // e2m1 1.0 in every nibble, e8m0 scale 127 (1.0) in every scale byte
    for (int i = threadIdx.x; i < 32768 / 4; i += kThreads) reinterpret_cast<uint32_t*>(smem)[i] = 0x22222222u;
    for (int i = threadIdx.x; i < 3072 / 4; i += kThreads) reinterpret_cast<uint32_t*>(sf)[i] = 0x7F7F7F7Fu;
    const uint32_t rank = cluster_ctarank();
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0)
    {
        mbar_init(&bar_loop, 1);
        mbar_init(&bar_end, 1);
        fence_mbar_init();
    }
    fence_proxy_async_smem();
    if (warp == 1)
    {
        tmem_alloc_pair(&tslot, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tb = tslot;
    const uint32_t sf_a = tb + 256, sf_b = sf_a + 8;
    if (threadIdx.x == 0 && rank == 0)
    {
#pragma unroll
        for (int q = 0; q < 2; ++q)
            tc_cp_32x128b_warpx4_pair(sf_a + 4 * q, make_smem_desc(smem_u32(sf + q * 512), 0, 128, 0));
#pragma unroll
        for (int c = 0; c < 4; ++c)
            tc_cp_32x128b_warpx4_pair(sf_b + 4 * c, make_smem_desc(smem_u32(sf + 1024 + c * 512), 0, 128, 0));
        const long long c0 = clock64();
        const unsigned long long t0 = globaltimer_ns();
        for (int g = 0; g < groups; ++g)
        {
#pragma unroll
            for (int j = 0; j < kMmaPerGroup; ++j)
            {
                const uint64_t ad = make_smem_desc(smem_u32(a) + j * 32, 16, 1024, 2);
                const uint64_t bd = make_smem_desc(smem_u32(b) + j * 2 * (128 * 16), 128 * 16, 128, 0);
                const uint32_t id = (uint32_t)(j & 1) * 2, q = (uint32_t)(j >> 1);
                tc_mma_mxf4_pair(tb, ad, bd, make_idesc_mxf4(256, 256, id, id), (sf_a + 4 * q) | (id << 30),
                                 (sf_b + 8 * q) | (id << 30), (g | j) ? 1u : 0u);
            }
            if ((g & 15) == 15) tc_commit_pair_mc(&bar_loop, 0x3);  // nobody waits: phases just advance
        }
        tc_commit_pair_mc(&bar_end, 0x3);
        const bool ok = mbar_wait(&bar_end, 0);
        g_cycles[blockIdx.x] = (unsigned long long)(clock64() - c0);
        g_ns[blockIdx.x] = globaltimer_ns() - t0;
        if (!ok) atomicExch(err, (unsigned)MBS_ERR_DEVICE_TIMEOUT);
    }
    else if (threadIdx.x == 0)
    {
        if (!mbar_wait(&bar_end, 0)) atomicExch(err, (unsigned)MBS_ERR_DEVICE_TIMEOUT);
    }
    tc_fence_before();
    __syncwarp();
    cluster_sync();  // no pair MMA can still target this CTA's TMEM
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tb, 512);
}

}  // namespace
}  // namespace probe
}  // namespace mbs

extern "C" int mbs_mxf4_peak_probe(int groups, double* tflops, double* cycles_per_mma, double* sm_mhz,
                                   void* stream)
{
    using namespace mbs::probe;
    mbs::clear_error();
    if (tflops == nullptr || cycles_per_mma == nullptr || sm_mhz == nullptr)
        return mbs::fail(MBS_ERR_INVALID_ARGUMENT, "mbs_mxf4_peak_probe: output pointers must be non-NULL");
    if (groups < 16 || groups > (1 << 24))
        return mbs::fail(MBS_ERR_INVALID_ARGUMENT, "mbs_mxf4_peak_probe: groups must be in [16, 2^24], got %d",
                         groups);
    mbs::DeviceInfo dev;
    int st = mbs::current_device(&dev);
    if (st) return st;
    const int grid = (dev.num_sms / 2) * 2 < kMaxCtas ? (dev.num_sms / 2) * 2 : kMaxCtas;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaFuncSetAttribute(mxf4_peak_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return mbs::cuda_fail(e, "cudaFuncSetAttribute (probe)");
    unsigned* err = mbs::device_error_word(dev.device);
    if (err == nullptr) return mbs::fail(MBS_ERR_CUDA, "device error word unavailable");
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if ((e = cudaEventCreate(&e0)) != cudaSuccess || (e = cudaEventCreate(&e1)) != cudaSuccess)
    {
        if (e0) cudaEventDestroy(e0);
        return mbs::cuda_fail(e, "cudaEventCreate (probe)");
    }
    mxf4_peak_probe_kernel<<<grid, kThreads, kSmem, s>>>(groups / 8 > 16 ? groups / 8 : 16, err);  // warm-up
    cudaEventRecord(e0, s);
    mxf4_peak_probe_kernel<<<grid, kThreads, kSmem, s>>>(groups, err);
    cudaEventRecord(e1, s);
    e = cudaEventSynchronize(e1);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (e != cudaSuccess) return mbs::cuda_fail(e, "mxf4 peak probe");
    unsigned long long cyc[kMaxCtas], ns[kMaxCtas];
    if ((e = cudaMemcpyFromSymbol(cyc, g_cycles, sizeof(unsigned long long) * grid)) != cudaSuccess ||
        (e = cudaMemcpyFromSymbol(ns, g_ns, sizeof(unsigned long long) * grid)) != cudaSuccess)
        return mbs::cuda_fail(e, "cudaMemcpyFromSymbol (probe)");
    unsigned code = 0;
    if ((e = cudaMemcpy(&code, err, sizeof(code), cudaMemcpyDeviceToHost)) != cudaSuccess)
        return mbs::cuda_fail(e, "cudaMemcpy (probe error word)");
    if (code != 0) return mbs::fail((int)code, "mbs_mxf4_peak_probe: a wait timed out on the device");
    double sum_cyc = 0, sum_ns = 0;
    for (int i = 0; i < grid; i += 2)
    {
        sum_cyc += (double)cyc[i];
        sum_ns += (double)ns[i];
    }
    const double mmas = (double)groups * kMmaPerGroup;
    *cycles_per_mma = sum_cyc / (grid / 2) / mmas;
    *sm_mhz = sum_ns > 0 ? sum_cyc / sum_ns * 1e3 : 0.0;
    const double flop = 2.0 * 256 * 256 * 64 * mmas * (grid / 2);
    *tflops = ms > 0 ? flop / (ms * 1e-3) / 1e12 : 0.0;
    return MBS_OK;
}
