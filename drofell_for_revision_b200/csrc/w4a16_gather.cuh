// Fused all-gather epilogue shared by the GEMV kernels (see GatherArgs).
#pragma once
#include "w4a16_internal.h"
#include "w4a16_ptx.cuh"

namespace w4a16 {

constexpr uint32_t kGatherSpinLimit = 1u << 22;  // x ~64 ns sleeps: well over a second
constexpr int kErrGatherTimeout = 128;

// Y[m, n] of this rank's columns into every rank's full Y (ga.world > 0), or into
// the local Y [M, N] (ga.world == 0).
__device__ __forceinline__ void out_store(const GatherArgs& ga, uint16_t* y, int N, int m, int n, uint16_t v) {
    if (ga.world == 0) {
        y[static_cast<size_t>(m) * N + n] = v;
        return;
    }
    const size_t off = static_cast<size_t>(m) * ga.ld + ga.col0 + n;
    for (int r = 0; r < ga.world; ++r) ga.y[r][off] = v;
}

// 8 outputs (16 bytes) of row m, columns n..n+7: into the local Y [M, N]
// (ga.world == 0), or into every rank's full Y (ld and col0 multiples of 8).
__device__ __forceinline__ void out_store16(const GatherArgs& ga, uint16_t* y, int N, int m, int n, uint4 v) {
    if (ga.world == 0) {
        *reinterpret_cast<uint4*>(y + static_cast<size_t>(m) * N + n) = v;
        return;
    }
    const size_t off = static_cast<size_t>(m) * ga.ld + ga.col0 + n;
    for (int r = 0; r < ga.world; ++r) *reinterpret_cast<uint4*>(ga.y[r] + off) = v;
}

// The GEMV and GEMM kernels only store (out_store, out_store16); completion is a separate one-warp kernel
// launched after them in the stream (gather_signal_kernel in w4a16_capi.cu): stream
// order guarantees the GEMV's stores, local and remote, are complete, so a single
// system-scope fence there orders them before this rank's epoch flags. (A fence in
// every CTA of the GEMV cost ~13 us per launch on B200; the signal kernel costs a
// launch.)
__device__ __forceinline__ void gather_signal_and_wait(const GatherArgs& ga, int* err) {
    const uint32_t ep = atomicAdd(ga.ctr + 1, 1u) + 1;  // this rank's epoch (atomic: no stale copy)
    __threadfence_system();
    for (int r = 0; r < ga.world; ++r) ptx::st_release_sys(ga.flags[r] + ga.rank, ep);
    for (int r = 0; r < ga.world; ++r) {
        uint32_t spins = 0;
        while (ptx::ld_acquire_sys(ga.my_flags + r) < ep) {
            if (++spins > kGatherSpinLimit) {
                if (err) atomicCAS(err, 0, kErrGatherTimeout);
                break;
            }
            __nanosleep(64);
        }
    }
}

}  // namespace w4a16
