// mma_sync.cu — warp-level mma.sync probes, kept so the reference's legacy
// tensor-core report keys (src/tensor_core.cu, src/tensor_core_extended.cu)
// resolve on B200.  These are the pre-Blackwell tensor path that the tcgen05
// GEMM (gemm.cu) and issue-rate probe (mma_rate.cu) supersede.
//
// Operands are constant ones; every MMA adds K to each accumulator element,
// so a chain of `iters` MMAs leaves K * iters (f32/s32 accumulators) and the
// result is checkable.  Latency: one warp, one dependent chain (unrolled by
// 8), %clock64 around it with the end read depending on the chain.
// Throughput: every warp runs kChains independent chains so the tensor pipe
// sees independent work from each warp.
#include <cuda_fp16.h>

#include "cmb_device.cuh"
#include "cmb_host.h"

namespace cmb {
namespace {

enum MmaKind { kTf32 = 0, kF16 = 1, kBf16 = 2, kE4m3 = 3, kS8 = 4 };

constexpr int kChains = 4;

// Accumulator registers of a kind: four f32 (tf32, bf16, e4m3), two
// packed f16x2 words (f16) or four s32 (s8).
template <int KIND>
struct Acc {
  float f[4] = {0.f, 0.f, 0.f, 0.f};
  uint32_t u[4] = {0u, 0u, 0u, 0u};
};

// One MMA of the given kind with all-ones operands: acc += 1 * 1 summed
// over K, i.e. every accumulator element grows by K.
template <int KIND>
__device__ __forceinline__ void mma_once(Acc<KIND> &c) {
  if constexpr (KIND == kTf32) {
    const uint32_t one = 0x3f800000u;  // tf32 1.0 (fp32 bit pattern)
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%11,%12,%13};"
        : "=f"(c.f[0]), "=f"(c.f[1]), "=f"(c.f[2]), "=f"(c.f[3])
        : "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "f"(c.f[0]), "f"(c.f[1]),
          "f"(c.f[2]), "f"(c.f[3]));
  } else if constexpr (KIND == kF16) {
    const uint32_t one = 0x3c003c00u;  // two fp16 1.0
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f16.f16.f16.f16 {%0,%1}, {%2,%3,%4,%5}, {%6,%7}, "
        "{%8,%9};"
        : "=r"(c.u[0]), "=r"(c.u[1])
        : "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "r"(c.u[0]), "r"(c.u[1]));
  } else if constexpr (KIND == kBf16) {
    const uint32_t one = 0x3f803f80u;  // two bf16 1.0
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%11,%12,%13};"
        : "=f"(c.f[0]), "=f"(c.f[1]), "=f"(c.f[2]), "=f"(c.f[3])
        : "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "f"(c.f[0]), "f"(c.f[1]),
          "f"(c.f[2]), "f"(c.f[3]));
  } else if constexpr (KIND == kE4m3) {
    const uint32_t one = 0x38383838u;  // four e4m3 1.0
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%11,%12,%13};"
        : "=f"(c.f[0]), "=f"(c.f[1]), "=f"(c.f[2]), "=f"(c.f[3])
        : "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "f"(c.f[0]), "f"(c.f[1]),
          "f"(c.f[2]), "f"(c.f[3]));
  } else {
    const uint32_t one = 0x01010101u;  // four s8 1
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%11,%12,%13};"
        : "=r"(c.u[0]), "=r"(c.u[1]), "=r"(c.u[2]), "=r"(c.u[3])
        : "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "r"(c.u[0]), "r"(c.u[1]),
          "r"(c.u[2]), "r"(c.u[3]));
  }
}

// Accumulator element 0 as a double (f16 accumulators hold half values).
template <int KIND>
__device__ __forceinline__ double acc_value(const Acc<KIND> &c) {
  if constexpr (KIND == kF16) return static_cast<double>(__half2float(__ushort_as_half(c.u[0] & 0xffffu)));
  else if constexpr (KIND == kS8) return static_cast<double>(static_cast<int>(c.u[0]));
  else return static_cast<double>(c.f[0]);
}

// A 32-bit value that depends on every accumulator register.
template <int KIND>
__device__ __forceinline__ uint32_t acc_dep(const Acc<KIND> &c) {
  if constexpr (KIND == kF16 || KIND == kS8) return c.u[0] ^ c.u[1] ^ c.u[2] ^ c.u[3];
  else return __float_as_uint(c.f[0]) ^ __float_as_uint(c.f[1]) ^ __float_as_uint(c.f[2]) ^
              __float_as_uint(c.f[3]);
}

// Dependent chain, unrolled by 8 so loop bookkeeping stays off the chain.
template <int KIND>
__global__ void k_mma_latency(int iters, uint64_t *cycles, double *value) {
  Acc<KIND> c;
  const uint64_t t0 = dev::clock64();
  int i = 0;
#pragma unroll 1
  for (; i + 8 <= iters; i += 8) {
#pragma unroll
    for (int u = 0; u < 8; ++u) mma_once<KIND>(c);
  }
#pragma unroll 1
  for (; i < iters; ++i) mma_once<KIND>(c);
  const uint64_t t1 = dev::clock64_after(acc_dep<KIND>(c));
  if (threadIdx.x == 0) {
    cycles[0] = t1 - t0;
    value[0] = acc_value<KIND>(c);
  }
}

template <int KIND>
__global__ void k_mma_throughput(int iters, double *value) {
  Acc<KIND> c[kChains];
#pragma unroll 1
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int k = 0; k < kChains; ++k) mma_once<KIND>(c[k]);
  }
  double s = 0.0;
#pragma unroll
  for (int k = 0; k < kChains; ++k) s += acc_value<KIND>(c[k]);
  if ((threadIdx.x & 31) == 0) value[(blockIdx.x * blockDim.x + threadIdx.x) >> 5] = s;
}

template <int KIND>
int launch(int latency, int iters, int blocks, int warps, uint64_t *cycles, double *value,
           cudaStream_t stream) {
  if (latency) k_mma_latency<KIND><<<1, 32, 0, stream>>>(iters, cycles, value);
  else k_mma_throughput<KIND><<<blocks, warps * 32, 0, stream>>>(iters, value);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}

int dispatch(int kind, int latency, int iters, int blocks, int warps, uint64_t *cycles,
             double *value, cudaStream_t stream) {
  switch (kind) {
    case kTf32: return launch<kTf32>(latency, iters, blocks, warps, cycles, value, stream);
    case kF16: return launch<kF16>(latency, iters, blocks, warps, cycles, value, stream);
    case kBf16: return launch<kBf16>(latency, iters, blocks, warps, cycles, value, stream);
    case kE4m3: return launch<kE4m3>(latency, iters, blocks, warps, cycles, value, stream);
    case kS8: return launch<kS8>(latency, iters, blocks, warps, cycles, value, stream);
    default: return fail(CMB_ERR_INVALID_ARG, "mma.sync probe: kind %d not in 0..4", kind);
  }
}

}  // namespace
}  // namespace cmb

using namespace cmb;

extern "C" int cmb_mma_sync_latency(int kind, int iters, uint64_t *cycles, double *value,
                                    cmb_stream_t stream) {
  if (cycles == nullptr || value == nullptr || iters < 1)
    return fail(CMB_ERR_INVALID_ARG, "cmb_mma_sync_latency: null output or iters < 1");
  return dispatch(kind, 1, iters, 1, 1, cycles, value, stream);
}

extern "C" int cmb_mma_sync_throughput(int kind, int iters, int blocks, int warps_per_block,
                                       double *values, cmb_stream_t stream) {
  if (values == nullptr || iters < 1 || blocks < 1 || warps_per_block < 1 || warps_per_block > 32)
    return fail(CMB_ERR_INVALID_ARG, "cmb_mma_sync_throughput: bad arguments");
  return dispatch(kind, 0, iters, blocks, warps_per_block, nullptr, values, stream);
}
