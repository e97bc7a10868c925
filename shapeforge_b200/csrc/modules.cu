// Loading and launching compiled candidate kernels: the harness half of the Candidate/Harness
// split on CUDA.  A candidate is a CUDA source with `extern "C" __global__` kernels taking the
// task's ABI tensors in order; the harness compiles it (nvcc -cubin for sm_100a), loads the image
// here and launches it with the geometry the candidate declared.  This replaces the Metal
// pipeline-state creation and dispatch of tcenv/backends/metal/runtime.py:306 (compile) and :593
// (run_pipeline) for candidate kernels.
#include "sf_common.cuh"

extern "C" int sf_module_load(const void* image, uint64_t size, void** module, char* err, uint64_t cap) {
    (void)size;
    if (!image || !module) return sf::fail(SF_EINVAL, err, cap, "sf_module_load: null image or output");
    cudaLibrary_t lib = nullptr;
    cudaError_t e = cudaLibraryLoadData(&lib, image, nullptr, nullptr, 0, nullptr, nullptr, 0);
    if (e != cudaSuccess) return sf::fail(SF_EDEVICE, err, cap, "cudaLibraryLoadData: %s", cudaGetErrorString(e));
    *module = (void*)lib;
    return SF_OK;
}

extern "C" int sf_module_unload(void* module, char* err, uint64_t cap) {
    if (!module) return sf::fail(SF_EINVAL, err, cap, "sf_module_unload: null module");
    cudaError_t e = cudaLibraryUnload((cudaLibrary_t)module);
    if (e != cudaSuccess) return sf::fail(SF_EDEVICE, err, cap, "cudaLibraryUnload: %s", cudaGetErrorString(e));
    return SF_OK;
}

extern "C" int sf_module_get_function(void* module, const char* name, void** function, char* err, uint64_t cap) {
    if (!module || !name || !function) return sf::fail(SF_EINVAL, err, cap, "sf_module_get_function: bad arguments");
    cudaKernel_t k = nullptr;
    cudaError_t e = cudaLibraryGetKernel(&k, (cudaLibrary_t)module, name);
    if (e != cudaSuccess) return sf::fail(SF_EINVAL, err, cap, "kernel %s not found in the module: %s", name, cudaGetErrorString(e));
    *function = (void*)k;
    return SF_OK;
}

extern "C" int sf_launch_kernel(void* function, uint32_t gx, uint32_t gy, uint32_t gz, uint32_t bx, uint32_t by, uint32_t bz,
                                uint32_t smem, void* stream, void** args, char* err, uint64_t cap) {
    if (!function) return sf::fail(SF_EINVAL, err, cap, "sf_launch_kernel: null function");
    if (!gx || !gy || !gz || !bx || !by || !bz) return sf::fail(SF_EINVAL, err, cap, "sf_launch_kernel: zero grid or block dimension");
    if ((uint64_t)bx * by * bz > 1024) return sf::fail(SF_EINVAL, err, cap, "sf_launch_kernel: more than 1024 threads per CTA");
    if (gy > 65535 || gz > 65535) return sf::fail(SF_EINVAL, err, cap, "sf_launch_kernel: grid y/z above 65535");
    const void* fn = (const void*)function;
    if (smem > 48 * 1024) {
        cudaError_t a = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (a != cudaSuccess) return sf::fail(SF_EINVAL, err, cap, "dynamic shared memory %u: %s", smem, cudaGetErrorString(a));
    }
    cudaError_t e = cudaLaunchKernel(fn, dim3(gx, gy, gz), dim3(bx, by, bz), args, smem, (cudaStream_t)stream);
    if (e != cudaSuccess) return sf::fail(SF_EDEVICE, err, cap, "cudaLaunchKernel: %s", cudaGetErrorString(e));
    return SF_OK;
}
