#pragma once

// Compilation-target macros shared by every kl header.
// Mirrors kernel_lib/include/kl/config.hpp:5-12, without the CUTLASS dependency: the
// sm_100-family test reads nvcc's own feature macros.

#if defined(__CUDACC__)
#define KL_HOST_DEVICE __host__ __device__ __forceinline__
#define KL_DEVICE __device__ __forceinline__
#else
#define KL_HOST_DEVICE inline
#define KL_DEVICE inline
#endif

// Defined in device passes that may emit sm_100-family instructions (tcgen05, TMEM, TMA pair loads).
// nvcc sets __CUDA_ARCH_FEAT_SM100_ALL for sm_100a and __CUDA_ARCH_FAMILY_SPECIFIC__ for sm_100f/103f.
#if defined(__CUDA_ARCH__) &&                                                        \
    (defined(__CUDA_ARCH_FEAT_SM100_ALL) || defined(__CUDA_ARCH_FEAT_SM103_ALL) ||   \
     (defined(__CUDA_ARCH_FAMILY_SPECIFIC__) && __CUDA_ARCH_FAMILY_SPECIFIC__ >= 1000 && \
      __CUDA_ARCH_FAMILY_SPECIFIC__ < 1100))
#define KL_ARCH_SM100 1
#endif
