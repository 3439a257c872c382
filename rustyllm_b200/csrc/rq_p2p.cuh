// rq_p2p.cuh -- layout of a rank's NVLink exchange region (CUDA IPC, mapped
// by every peer) and its memory-order primitives, shared by the standalone
// one-shot all-reduce (rq_tp.cu) and the matvec pipeline's fused
// all-reduce epilogue (rq_mv_pipe.cu).
//
// Region: data [2 parities][kP2PCap bytes] | flags [2][kP2PFlagCTAs][kP2PMaxWorld]
// u32 | control words (epoch, done, err).  A call with epoch e uses parity
// e & 1; CTA c of rank r release-stores e + 1 into flags[parity][c][r] of
// every peer once its slice is in its own data buffer; the last CTA to
// finish bumps the epoch.
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace rq {

constexpr int kP2PMaxWorld = 8;
constexpr int kP2PFlagCTAs = 160;  // flag slots per parity: up to one CTA per SM
constexpr size_t kP2PCap = 4u << 20;  // bytes per buffer parity
constexpr size_t kP2PFlagsOff = 2 * kP2PCap;
constexpr size_t kP2PCtlOff = kP2PFlagsOff + 2 * (size_t)kP2PFlagCTAs * kP2PMaxWorld * 4;
constexpr size_t kP2PBytes = kP2PCtlOff + 256;

struct P2PArgs {
    uint8_t* base[kP2PMaxWorld];  // every rank's exchange region (own included), in this process
    int world, rank;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

}  // namespace rq
