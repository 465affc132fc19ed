// Fused all-gather epilogue shared by the GEMV kernels (see GatherArgs).
#pragma once
#include "w4a16_internal.h"
#include "w4a16_ptx.cuh"

namespace w4a16 {

constexpr uint32_t kGatherSpinLimit = 1u << 23;  // x ~32 ns sleeps: well over a second
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
// One warp; lane r < world talks to rank r, so the flag stores and the waits of all
// ranks run side by side: one system-scope fence (the stores of the kernel before
// are complete, griddepcontrol.wait), then relaxed flag stores, relaxed polls, and one
// acquire fence once every rank's flag has arrived.
__device__ __forceinline__ void gather_signal_and_wait(const GatherArgs& ga, int* err) {
    const int lane = static_cast<int>(threadIdx.x & 31);
    uint32_t ep = 0;
    if (lane == 0) ep = atomicAdd(ga.ctr + 1, 1u) + 1;  // this rank's epoch (atomic: no stale copy)
    ep = __shfl_sync(0xffffffffu, ep, 0);
    __threadfence_system();
    if (lane < ga.world) {
        ptx::st_relaxed_sys(ga.flags[lane] + ga.rank, ep);
        uint32_t spins = 0;
        while (ptx::ld_relaxed_sys(ga.my_flags + lane) < ep) {
            if (++spins > kGatherSpinLimit) {
                if (err) atomicCAS(err, 0, kErrGatherTimeout);
                break;
            }
            __nanosleep(32);
        }
    }
    __syncwarp();
    ptx::fence_acq_rel_sys();  // the peers' rows, written before their flags, are visible from here on
}

}  // namespace w4a16
