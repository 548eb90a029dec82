// Shared pieces of the library's tcgen05 / TMA kernels (inmap.cu, readout.cu): mbarriers with bounded
// waits, 2-D TMA loads, the shared-memory descriptor of a K-major SWIZZLE_128B float16 operand tile, the
// kind::f16 instruction descriptor, and the tensor-map encoder.
#pragma once

#include <cudaTypedefs.h>

#include "common.cuh"

namespace afb {
namespace tc {

constexpr uint32_t kWaitLimit = 1u << 22;       // polls of a bounded mbarrier wait before it gives up
constexpr int kBK = 64;                         // 64 float16 = one 128-byte swizzle row
constexpr int kMmaK = 16;                       // K of one tcgen05.mma kind::f16

// Instruction descriptor of tcgen05.mma kind::f16: D float32 (bits 4-5 = 1), A and B float16 (bits 7-9,
// 10-12 = 0), both K-major (bits 15, 16 = 0), N >> 3 in bits 17-22, M >> 4 in bits 24-28.
constexpr uint32_t idesc_f16(int m, int n) { return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24); }

// Shared-memory descriptor of a K-major SWIZZLE_128B operand tile whose rows are 128 bytes and whose
// 8-row groups are 1024 bytes apart: start address >> 4 (bits 0-13), leading byte offset 16 B >> 4
// (bits 16-29, unused by this layout), stride byte offset 1024 B >> 4 (bits 32-45), descriptor version 1
// (bits 46-47), swizzle mode 2 = 128 B (bits 61-63).  The tile base is 1024-byte aligned.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}

__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t it = 0; it < kWaitLimit; ++it) {
        uint32_t ok;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
        if (ok) return true;
    }
    return false;
}
__device__ __forceinline__ void bar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}\n" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void fail(int *status, int code) {
    if (status) atomicOr(status, code);
}

__device__ __forceinline__ void tma_load(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n"
                 ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar) : "memory");
}

// D (TMEM) (+)= A B^T for one K = 16 step; accumulate = 0 overwrites D.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
                 ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// The mbarrier fires once every MMA this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}

// 32 consecutive float32 columns of this warp's 32 TMEM lanes (lane quarter by warp), one per register.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
                 " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                   "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                   "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// cuTensorMapEncodeTiled from the driver (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// A K-major float16 operand: rows x k_dim elements, row stride ld elements (a multiple of 8), boxes of
// box_rows x 64, SWIZZLE_128B; rows and columns past the extents read as zero.
void encode_operand(CUtensorMap *map, const void *base, int64_t rows, int64_t k_dim, int64_t ld, uint32_t box_rows);

}  // namespace tc
}  // namespace afb
