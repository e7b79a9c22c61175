/* TEST INFRASTRUCTURE -- the CUDA/HIP vocabulary the reference kernel file uses, mapped
 * onto host C++ so that file compiles unchanged with g++ and its kernels run on the CPU.
 *
 * A "launch" runs the grid block by block. Within a block, kernels that never call
 * __syncthreads() run their threads one after another on the calling thread; kernels
 * that do (the per-filter reductions) get one std::thread per CUDA thread meeting at a
 * std::barrier, so shared memory and barriers behave as on a device. __shared__ arrays
 * become function-local statics: one copy, seen by every thread of the block that is
 * running, which is what shared memory is while blocks run one at a time. */
#ifndef DNB_HIP_HOST_SHIM_H
#define DNB_HIP_HOST_SHIM_H

#include <barrier>
#include <cmath>
#include <cstdint>

struct dnb_dim3 {
    unsigned x, y, z;
};

extern thread_local dnb_dim3 dnb_thread_idx;
extern thread_local dnb_dim3 dnb_block_idx;
extern dnb_dim3 dnb_block_dim;
extern dnb_dim3 dnb_grid_dim;
extern std::barrier<> *dnb_block_barrier;

#define threadIdx dnb_thread_idx
#define blockIdx dnb_block_idx
#define blockDim dnb_block_dim
#define gridDim dnb_grid_dim

#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __shared__ alignas(16) static
#define __align__(n)
#define __launch_bounds__(...)
#define __syncthreads() dnb_block_barrier->arrive_and_wait()

/* CUDA's integer min/max device overloads (used by col2im_kernel) */
inline int min(int a, int b) { return a < b ? a : b; }
inline int max(int a, int b) { return a > b ? a : b; }

struct float4 {
    float x, y, z, w;
};

#endif
