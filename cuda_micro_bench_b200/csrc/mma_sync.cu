// mma_sync.cu — warp-level mma.sync probes, kept so the reference's legacy
// tensor-core report keys (src/tensor_core.cu, src/tensor_core_extended.cu)
// resolve on B200.  These are the pre-Blackwell tensor path that the tcgen05
// GEMM (gemm.cu) and issue-rate probe (mma_rate.cu) supersede.
//
// Operands are constant ones; every MMA adds K to each accumulator element,
// so a chain of `iters` MMAs leaves K * iters (f32/s32 accumulators) and the
// result is checkable.  Latency: one warp, one dependent chain, %clock64
// around it with the end read depending on the chain.  Throughput: every
// warp runs kChains independent chains so the tensor pipe sees independent
// work from each warp.
#include <cuda_fp16.h>

#include "cmb_device.cuh"
#include "cmb_host.h"

namespace cmb {
namespace {

enum MmaKind { kTf32 = 0, kF16 = 1, kBf16 = 2, kE4m3 = 3, kS8 = 4 };

constexpr int kChains = 4;

// One MMA of the given kind: c (4 x 32-bit accumulator registers; for f16
// only c[0..1] are used) += a * b with all-ones operands.
template <int KIND>
__device__ __forceinline__ void mma_once(uint32_t (&c)[4]) {
  if constexpr (KIND == kTf32) {
    const uint32_t one = 0x3f800000u;  // tf32 1.0 (fp32 bit pattern)
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "r"(one));
  } else if constexpr (KIND == kF16) {
    const uint32_t one = 0x3c003c00u;  // two fp16 1.0
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f16.f16.f16.f16 {%0,%1}, {%2,%3,%4,%5}, {%6,%7}, "
        "{%0,%1};"
        : "+r"(c[0]), "+r"(c[1])
        : "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "r"(one));
  } else if constexpr (KIND == kBf16) {
    const uint32_t one = 0x3f803f80u;  // two bf16 1.0
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "r"(one));
  } else if constexpr (KIND == kE4m3) {
    const uint32_t one = 0x38383838u;  // four e4m3 1.0
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "r"(one));
  } else {
    const uint32_t one = 0x01010101u;  // four s8 1
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(one), "r"(one), "r"(one), "r"(one), "r"(one), "r"(one));
  }
}

// Accumulator element 0 as a double (f16 accumulators hold half values).
template <int KIND>
__device__ __forceinline__ double acc_value(const uint32_t (&c)[4]) {
  if constexpr (KIND == kF16) return static_cast<double>(__half2float(__ushort_as_half(c[0] & 0xffffu)));
  else if constexpr (KIND == kS8) return static_cast<double>(static_cast<int>(c[0]));
  else return static_cast<double>(__uint_as_float(c[0]));
}

template <int KIND>
__global__ void k_mma_latency(int iters, uint64_t *cycles, double *value) {
  uint32_t c[4] = {0, 0, 0, 0};
  const uint64_t t0 = dev::clock64();
#pragma unroll 1
  for (int i = 0; i < iters; ++i) mma_once<KIND>(c);
  const uint64_t t1 = dev::clock64_after(c[0] ^ c[1]);
  if (threadIdx.x == 0) {
    cycles[0] = t1 - t0;
    value[0] = acc_value<KIND>(c);
  }
}

template <int KIND>
__global__ void k_mma_throughput(int iters, double *value) {
  uint32_t c[kChains][4] = {};
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
