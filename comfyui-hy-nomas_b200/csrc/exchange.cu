// Arrival wait of the sequence-parallel K/V exchange: the copy engines push every rank's K and V slices into the
// peers' buffers and then write a 32-bit block counter into each peer's flag array (a memory fence precedes the
// write). Attention on a rank may start once every peer's flags have reached this block's counter.
//
// One warp polls the flags with system-scope acquire loads, so the pushed data is visible to the kernels that
// follow on the stream. The wait is bounded: past `limit_ns` it records HN_DEVERR_TIMEOUT in the stream's error
// word and returns, so a peer that never arrives leaves a usable context and an error the host reads.
#include <cstdint>

#include "hn_common.cuh"
#include "hn_kernels.h"

namespace hn {

__global__ void k_wait_flags(const uint32_t *flags, int groups, int count, int group_stride, int skip, uint32_t value,
                             uint64_t limit_ns, int *err) {
    const uint64_t t0 = globaltimer_ns();
    const int total = groups * count;
    bool timed_out = false;
    for (int i = threadIdx.x; i < total && !timed_out; i += blockDim.x) {
        const int g = i / count, c = i - g * count;
        if (c == skip) continue;
        const uint32_t *f = flags + (int64_t)g * group_stride + c;
        while (true) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
            if ((int32_t)(v - value) >= 0) break;      // wrap-safe "v >= value"
            if (globaltimer_ns() - t0 > limit_ns) {
                atomicOr(err, HN_DEVERR_TIMEOUT);
                timed_out = true;
                break;
            }
            __nanosleep(256);
        }
    }
    __syncwarp();
}

cudaError_t launch_wait_flags(const uint32_t *flags, int groups, int count, int group_stride, int skip,
                              uint32_t value, uint32_t timeout_us, cudaStream_t st) {
    int *err = nullptr;
    cudaError_t e = device_error_word(err_slot(st), &err);
    if (e != cudaSuccess) return e;
    k_wait_flags<<<1, 32, 0, st>>>(flags, groups, count, group_stride, skip, value, (uint64_t)timeout_us * 1000ull,
                                   err);
    return cudaGetLastError();
}

} // namespace hn
