/* Build manifest for compiling the reference's bench/framework sources on an
 * x86 host as the parity checker (oracle/_ref).  The reference generates this
 * header from bench/framework/build_manifest.h.in with CMake; the checker
 * build only needs the constants to exist.  No kernel is registered in the
 * checker, so the platform name is informational. */
#ifndef PFNG_BENCH_BUILD_MANIFEST_H
#define PFNG_BENCH_BUILD_MANIFEST_H

#include <array>
#include <cstddef>
#include <string_view>

namespace pfng::bench {

inline constexpr std::string_view kBuildTargetPlatform = "x86-host-checker";
inline constexpr std::string_view kBuildPlatformDisplayName = "x86 host (parity checker)";
inline constexpr std::string_view kBuildTargetArch = "x86-64";
inline constexpr std::string_view kBuildTargetTune = "generic";
inline constexpr std::string_view kBuildCompiler = "g++";
inline constexpr std::string_view kBuildCompilerVersion = "host";
inline constexpr size_t kBuildFirstCpu = 0;
inline constexpr size_t kBuildLastCpu = 0;
inline constexpr size_t kBuildMaxThreads = 1;
inline constexpr std::array<std::string_view, 1> kBuildDeviceTreeCompatibles = {"none"};

} // namespace pfng::bench

#endif
