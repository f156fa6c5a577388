// platform_cuda.cpp -- runtime platform detection for the nvidia-b200 build
// of the reference's bench framework.
//
// The reference identifies its RISC-V boards by their Device Tree
// `compatible` strings (bench/framework/platform.cpp:62-83); a GPU host has
// no such entry for its accelerator.  For the nvidia-b200 build,
// detect_runtime_platform() asks the CUDA runtime instead: the platform is
// NvidiaB200 when the current device has compute capability 10.0.  The
// result has the reference's shape -- model = the device name, compatibles =
// "cuda,sm_<major><minor>", error text when no such device is present -- so
// --platform-info, --check-platform and the run-time platform check of
// bench/main.cpp work unchanged.
#include "platform.h"

#include <cuda_runtime.h>

#include <string>

namespace pfng::bench {

PlatformDetectionResult detect_cuda_platform() {
    PlatformDetectionResult result;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        result.error = std::string("no CUDA device: ") + (e != cudaSuccess ? cudaGetErrorString(e) : "count is 0");
        cudaGetLastError();
        return result;
    }
    int device = 0;
    cudaDeviceProp prop{};
    if ((e = cudaGetDevice(&device)) != cudaSuccess || (e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) {
        result.error = std::string("cudaGetDeviceProperties: ") + cudaGetErrorString(e);
        return result;
    }
    result.model = prop.name;
    result.compatibles.push_back("cuda,sm_" + std::to_string(prop.major * 10 + prop.minor));
    if (prop.major == 10 && prop.minor == 0)
        result.platform = PlatformId::NvidiaB200;
    else
        result.error = "CUDA device " + result.model + " is not compute capability 10.0 (B200)";
    return result;
}

}  // namespace pfng::bench
