/*
 * Host-only stand-in for the HIP runtime header, used ONLY to compile the
 * reference's q4rdna_gemv_bench.hip as plain C++ so that its CPU functions
 * (half_to_float, reference_q4_rdna) can be called as a checker.  The GPU
 * kernels in that file are compiled as dead host functions and never run;
 * every runtime call below is a no-op that reports failure.
 */
#pragma once
#include <cstddef>
#include <cstdint>

#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __shared__ static
#define __launch_bounds__(...)

struct q4shim_dim3 { unsigned x, y, z; q4shim_dim3(unsigned a = 1, unsigned b = 1, unsigned c = 1) : x(a), y(b), z(c) {} };
typedef q4shim_dim3 dim3;
static q4shim_dim3 threadIdx, blockIdx, blockDim, gridDim;
static inline void __syncwarp(unsigned = 0xffffffffu) {}
static inline void __syncthreads() {}

typedef int hipError_t;
enum { hipSuccess = 0, hipErrorNotSupported = 801 };
enum hipMemcpyKind { hipMemcpyHostToDevice = 1, hipMemcpyDeviceToHost = 2 };
typedef void *hipEvent_t;
struct hipDeviceProp_t { char name[256]; char gcnArchName[256]; };
static inline const char *hipGetErrorString(hipError_t) { return "HIP runtime not available (host shim)"; }
static inline hipError_t hipSetDevice(int) { return hipErrorNotSupported; }
static inline hipError_t hipMalloc(void *, size_t) { return hipErrorNotSupported; }
template <typename T> static inline hipError_t hipMalloc(T **, size_t) { return hipErrorNotSupported; }
static inline hipError_t hipFree(void *) { return hipErrorNotSupported; }
static inline hipError_t hipMemcpy(void *, const void *, size_t, int) { return hipErrorNotSupported; }
static inline hipError_t hipDeviceSynchronize() { return hipErrorNotSupported; }
static inline hipError_t hipEventCreate(hipEvent_t *) { return hipErrorNotSupported; }
static inline hipError_t hipEventRecord(hipEvent_t, void * = nullptr) { return hipErrorNotSupported; }
static inline hipError_t hipEventSynchronize(hipEvent_t) { return hipErrorNotSupported; }
static inline hipError_t hipEventElapsedTime(float *, hipEvent_t, hipEvent_t) { return hipErrorNotSupported; }
static inline hipError_t hipEventDestroy(hipEvent_t) { return hipErrorNotSupported; }
static inline hipError_t hipGetDeviceProperties(hipDeviceProp_t *, int) { return hipErrorNotSupported; }
#define hipLaunchKernelGGL(kernel, grid, block, shmem, stream, ...) ((void)0)
