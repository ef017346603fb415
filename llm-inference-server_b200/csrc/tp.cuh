// tp.cuh -- synchronisation of head-sharded ranks (one GPU each) over NVLink.
//
// A head-sharded decode step stores each rank's attention output slice into
// every rank's gathered buffer (attention epilogue, OutSpec with n > 0), then
// meets at this barrier before the gathered buffer is read.  Flags live in
// each rank's own memory; peers write them through IPC-mapped addresses with
// release stores at system scope and the owner polls them with acquire loads.
// Epochs grow by one per step (tp_epoch_bump), so a flag that is already
// ahead (a peer one barrier further on) also satisfies the wait.
#pragma once

#include "b2_common.cuh"

namespace b2 {

constexpr uint64_t kTpWaitLimitNs = 2000000000ull;  // default 2 s: a peer that does not arrive is an error

__global__ void __launch_bounds__(32) tp_barrier_kernel(uint32_t* local_flags, uint32_t* const* peer_flags, int rank,
                                                        int n, const uint32_t* epoch_ptr, int slot, uint64_t limit_ns) {
    const int t = threadIdx.x;
    const uint32_t epoch = *epoch_ptr;
    // Every store this GPU issued before (the attention epilogue's stores into
    // peers' gathered buffers, in the kernel before this one) is ordered
    // before the flags below at system scope.
    __threadfence_system();
    __syncwarp();
    if (t < n) {
        uint32_t* f = peer_flags[t] + static_cast<size_t>(slot) * n + rank;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(epoch) : "memory");
    }
    // A barrier of this device already gave up (a peer that stopped, seen by
    // an earlier layer of the step): the step is failed, so do not wait again.
    const bool given_up = (*reinterpret_cast<volatile unsigned int*>(&g_device_errors) & B2_DEVERR_TIMEOUT) != 0u;
    if (t < n && !given_up) {
        const uint32_t* mine = local_flags + static_cast<size_t>(slot) * n + t;
        const uint64_t t0 = global_timer_ns();
        bool ok = true;
        for (uint32_t it = 0;; ++it) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
            if (static_cast<int>(v - epoch) >= 0) break;  // reached (wrap-safe)
            if ((it & 63u) == 63u && global_timer_ns() - t0 > limit_ns) {
                ok = false;
                break;
            }
            __nanosleep(100);
        }
        if (!ok) flag_error(B2_DEVERR_TIMEOUT);
    }
    __syncwarp();
}

__global__ void tp_epoch_bump_kernel(uint32_t* epoch) {
    if (threadIdx.x == 0) *epoch += 1u;
}

// Sets bits in the device error word from the host's side of a test: error
// propagation is exercised without making any kernel fail.
__global__ void raise_device_error_kernel(unsigned int bits) {
    if (threadIdx.x == 0) flag_error(bits);
}

}  // namespace b2
