# Platform profile for an NVIDIA B200 (sm_100a) host, the format of the
# reference's platforms/*.cmake (read by cmake/PlatformConfig.cmake).  The
# kernels declared for this platform run on the GPU through libpfng_b200.so;
# the host side (CLI, registry, llama_reference verification) is built for
# the x86-64 host.  PFNG_PLATFORM_KIND "cuda" switches off the RISC-V-only
# steps of the build (cross-compiler checks, RVV assembly listings,
# machine-benchmarks) -- see the overlay edits in integration/build_pfng_bench.py.
set(PFNG_PLATFORM_ID "nvidia-b200")
set(PFNG_PLATFORM_DISPLAY_NAME "NVIDIA B200 (sm_100a)")
set(PFNG_PLATFORM_KIND "cuda")
set(PFNG_PLATFORM_ARCH "x86-64+sm_100a")
set(PFNG_PLATFORM_TUNE "generic")
set(PFNG_PLATFORM_COMPILE_DEFINITIONS PFNG_PLATFORM_NVIDIA_B200)
# No Device Tree on a GPU host: the runtime check asks the CUDA driver for a
# compute-capability 10.0 device instead (bench/framework/platform_cuda.cpp).
set(PFNG_PLATFORM_DEVICE_TREE_COMPATIBLES "cuda,sm_100")
set(PFNG_PLATFORM_FIRST_CPU 0)
set(PFNG_PLATFORM_LAST_CPU 255)
set(PFNG_PLATFORM_MAX_THREADS 256)
set(PFNG_PLATFORM_KERNEL_COMPILE_OPTIONS -O2)
set(PFNG_PLATFORM_FIXED_VLEN_COMPILE_OPTIONS -O2)
# Where libpfng_b200.so and its headers live (this repository's root).
if(NOT DEFINED PFNG_B200_ROOT)
    message(FATAL_ERROR "nvidia-b200: pass -DPFNG_B200_ROOT=<B200 library checkout>")
endif()
