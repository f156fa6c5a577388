"""Builds the reference's own pfng-bench CLI with the three B200 kernel IDs.

    python integration/build_pfng_bench.py --reference <reference checkout> [--out <binary>]

The reference is read-only input: it is copied to a temporary directory,
the overlay is applied to the copy, pfng-bench is compiled from it with g++,
and the copy is deleted.  Only the binary is kept
(integration/_build/pfng-bench by default, git-ignored; it finds
libpfng_b200.so through a relative rpath, so it travels with the tree).

The overlay is what a maintainer adds to the reference to get a B200 platform
(each edit below names the reference file and what it changes):
  * platforms/nvidia-b200.cmake                 -- the platform profile
  * kernels/{q4_0-q8_0,q4_K-q8_K,iq2_xxs-q8_K}-B200/CMakeLists.txt
                                                -- pfng_declare_kernel (cmake/Kernel.cmake)
  * bench/framework/platform.h / platform.cpp   -- PlatformId::NvidiaB200, its name,
                                                   and the CUDA detector (platform_cuda.cpp)
  * kernels/common/adapter_common.h             -- the register_*_b200 declarations
  * kernels/CMakeLists.txt, CMakeLists.txt, cmake/PlatformConfig.cmake,
    kernels/common/CMakeLists.txt               -- the RISC-V-only build steps skipped
                                                   for PFNG_PLATFORM_KIND "cuda"
The compile below does what the CMake target pfng-bench (CMakeLists.txt:
add_executable(pfng-bench ...)) does for that platform -- the same source
list, build_manifest.h from bench/framework/build_manifest.h.in with the
profile's values, builtin_kernels.cpp as cmake/Kernel.cmake's
pfng_generate_builtin_kernels writes it -- without running CMake.  bench/
main.cpp, the registry, run_benchmark's verification and timing and
llama_reference are the reference's sources, unmodified.
"""
from __future__ import annotations

import argparse
import os
import pathlib
import shutil
import subprocess
import sys
import tempfile

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent
OVERLAY = HERE / "overlay"
CUDA = pathlib.Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
KERNELS = (("q4_0-q8_0-B200", "register_q4_0_q8_0_b200"),
           ("q4_K-q8_K-B200", "register_q4_K_q8_K_b200"),
           ("iq2_xxs-q8_K-B200", "register_iq2_xxs_q8_K_b200"))
PROFILE = {  # the values of overlay/platforms/nvidia-b200.cmake the manifest needs
    "PFNG_PLATFORM_ID": "nvidia-b200",
    "PFNG_PLATFORM_DISPLAY_NAME": "NVIDIA B200 (sm_100a)",
    "PFNG_PLATFORM_ARCH": "x86-64+sm_100a",
    "PFNG_PLATFORM_TUNE": "generic",
    "PFNG_PLATFORM_FIRST_CPU": "0",
    "PFNG_PLATFORM_LAST_CPU": "255",
    "PFNG_PLATFORM_MAX_THREADS": "256",
    "PFNG_PLATFORM_COMPATIBLE_INITIALIZERS": '"cuda,sm_100"',
}


def edit(path: pathlib.Path, anchor: str, replacement: str) -> None:
    """Replace the one occurrence of `anchor` in `path`; fail loudly if the reference changed."""
    text = path.read_text()
    if text.count(anchor) != 1:
        raise SystemExit(f"overlay: {path} does not contain exactly one {anchor!r}")
    path.write_text(text.replace(anchor, replacement))


def apply_overlay(tree: pathlib.Path) -> None:
    fw = tree / "bench" / "framework"
    # PlatformId::NvidiaB200 and the CUDA detector's declaration (platform.h:11-16, :28-33)
    edit(fw / "platform.h", "    SpacemitK3A100,\n", "    SpacemitK3A100,\n    NvidiaB200,\n")
    edit(fw / "platform.h", "bool verify_runtime_platform(",
         "PlatformDetectionResult detect_cuda_platform();\nbool verify_runtime_platform(")
    # its name both ways (platform.cpp:38-56) and detection through CUDA (platform.cpp:62-83)
    edit(fw / "platform.cpp", '    case PlatformId::Unknown: return "unknown";',
         '    case PlatformId::NvidiaB200: return "nvidia-b200";\n    case PlatformId::Unknown: return "unknown";')
    edit(fw / "platform.cpp", "        return PlatformId::SpacemitK3A100;\n",
         '        return PlatformId::SpacemitK3A100;\n    if (name == "nvidia-b200") return PlatformId::NvidiaB200;\n')
    edit(fw / "platform.cpp", "    PlatformDetectionResult result;\n    const std::string compatible",
         "    if (build_target_platform() == PlatformId::NvidiaB200) return detect_cuda_platform();\n"
         "    PlatformDetectionResult result;\n    const std::string compatible")
    # the registration functions (kernels/common/adapter_common.h:76-96)
    edit(tree / "kernels" / "common" / "adapter_common.h", "void register_builtin_kernels();",
         "".join(f"void {fn}();\n" for _, fn in KERNELS) + "void register_builtin_kernels();")
    # new files: the profile, the kernel declarations, the detector
    shutil.copytree(OVERLAY, tree, dirs_exist_ok=True)
    # CMake: the kernel directories, and the RISC-V-only steps skipped for a CUDA platform
    with open(tree / "kernels" / "CMakeLists.txt", "a") as f:
        f.write("".join(f"add_subdirectory({kid})\n" for kid, _ in KERNELS))
    top = tree / "CMakeLists.txt"
    edit(top, "if(NOT CMAKE_TOOLCHAIN_FILE)\n",
         'if(PFNG_TARGET_PLATFORM MATCHES "^nvidia-")\n    set(PFNG_PLATFORM_KIND cuda)\nendif()\n'
         'if(NOT CMAKE_TOOLCHAIN_FILE AND NOT PFNG_PLATFORM_KIND STREQUAL "cuda")\n')
    edit(top, "   AND NOT DEFINED ENV{CXX})", '   AND NOT DEFINED ENV{CXX}\n   AND NOT PFNG_PLATFORM_KIND STREQUAL "cuda")')
    edit(top, "add_subdirectory(machine-benchmarks)\n",
         'if(NOT PFNG_PLATFORM_KIND STREQUAL "cuda")\n    add_subdirectory(machine-benchmarks)\nendif()\n')
    edit(top, "target_link_options(pfng-bench PRIVATE -fopenmp=libomp)\n",
         'if(PFNG_PLATFORM_KIND STREQUAL "cuda")\n'
         '    target_sources(pfng-bench PRIVATE bench/framework/platform_cuda.cpp)\n'
         '    find_package(CUDAToolkit REQUIRED)\n'
         '    target_link_libraries(pfng-bench PRIVATE CUDA::cudart)\n'
         'else()\n    target_link_options(pfng-bench PRIVATE -fopenmp=libomp)\nendif()\n')
    edit(top, "add_pfng_assembly(bench/main.cpp main)\n",
         'if(NOT PFNG_PLATFORM_KIND STREQUAL "cuda")\nadd_pfng_assembly(bench/main.cpp main)\n')
    edit(top, "add_dependencies(assembly ${PFNG_ASM_TARGETS})\n",
         "add_dependencies(assembly ${PFNG_ASM_TARGETS})\nendif()\n")
    cfg = tree / "cmake" / "PlatformConfig.cmake"
    edit(cfg, 'if(NOT CMAKE_SYSTEM_PROCESSOR MATCHES "[Rr][Ii][Ss][Cc][Vv]")',
         'if(NOT PFNG_PLATFORM_KIND STREQUAL "cuda")\nif(NOT CMAKE_SYSTEM_PROCESSOR MATCHES "[Rr][Ii][Ss][Cc][Vv]")')
    edit(cfg, 'message(STATUS "PFNG target platform: ${PFNG_PLATFORM_ID}")',
         'endif()\nmessage(STATUS "PFNG target platform: ${PFNG_PLATFORM_ID}")')
    common = tree / "kernels" / "common" / "CMakeLists.txt"
    edit(common, "    ../iq2_xxs-q8_K-RVV-common/implementations/rvv-vlen256/iq2_xxs_adapter.cpp\n)",
         ')\nif(NOT PFNG_PLATFORM_KIND STREQUAL "cuda")\n    pfng_add_kernel_sources(SOURCES\n'
         '        ../iq2_xxs-q8_K-RVV-common/implementations/rvv-vlen256/iq2_xxs_adapter.cpp)\nendif()')


def generate(tree: pathlib.Path, cxx: str) -> pathlib.Path:
    """build/generated/{build_manifest.h, builtin_kernels.cpp} as the CMake build writes them."""
    gen = tree / "build" / "generated"
    gen.mkdir(parents=True)
    version = subprocess.run([cxx, "-dumpfullversion"], capture_output=True, text=True).stdout.strip() or "unknown"
    values = dict(PROFILE, CMAKE_CXX_COMPILER=shutil.which(cxx) or cxx, CMAKE_CXX_COMPILER_VERSION=version)
    text = (tree / "bench" / "framework" / "build_manifest.h.in").read_text()
    for key, value in values.items():
        text = text.replace(f"@{key}@", value)
    if "@" in text:
        raise SystemExit("overlay: build_manifest.h.in has a placeholder this script does not fill")
    (gen / "build_manifest.h").write_text(text)
    body = "".join(f"    {fn}();\n" for _, fn in KERNELS)
    (gen / "builtin_kernels.cpp").write_text(
        '#include "adapter_common.h"\n\nnamespace pfng::bench::adapters {\nvoid register_builtin_kernels() {\n'
        + body + "}\n} // namespace pfng::bench::adapters\n")
    return gen


def build(reference: pathlib.Path, out: pathlib.Path, cxx: str = "g++") -> None:
    lib = ROOT / "qgemm-perf-framework-ng_b200" / "libpfng_b200.so"
    if not lib.exists():
        raise SystemExit(f"{lib} is not built (make -C qgemm-perf-framework-ng_b200)")
    with tempfile.TemporaryDirectory(prefix="pfng-overlay-") as tmp:
        tree = pathlib.Path(tmp) / "reference"
        # the checkout without version control and build trees (top-level build* directories)
        skip = lambda d, names: [n for n in names if n == ".git" or (d == str(reference) and n.startswith("build"))]
        shutil.copytree(reference, tree, ignore=skip)
        apply_overlay(tree)
        gen = generate(tree, cxx)
        sources = [tree / p for p in (
            "bench/main.cpp", "bench/framework/aligned_new.cpp", "bench/framework/kernel_registry.cpp",
            "bench/framework/benchmark.cpp", "bench/framework/platform.cpp",
            "bench/framework/platform_cuda.cpp", "bench/llama_reference/llama_reference.cpp",
            "kernels/common/adapter_common.cpp", "kernels/common/tcm_arena.cpp")]
        sources += [gen / "builtin_kernels.cpp", ROOT / "qgemm-perf-framework-ng_b200" / "host" / "b200_kernels.cpp"]
        includes = [tree / "include", tree / "bench", tree / "bench" / "framework", tree / "bench" / "llama_reference",
                    tree / "kernels" / "common", gen, ROOT / "include", ROOT / "qgemm-perf-framework-ng_b200" / "host",
                    CUDA / "include"]
        out.parent.mkdir(parents=True, exist_ok=True)
        rpath = os.path.relpath(lib.parent, out.parent)
        cmd = [cxx, "-O2", "-std=c++20", "-fopenmp", "-DPFNG_PLATFORM_NVIDIA_B200",
               "-DPFNG_B200_PLATFORM=pfng::bench::PlatformId::NvidiaB200",
               *[f"-I{p}" for p in includes], *map(str, sources), "-o", str(out),
               f"-L{lib.parent}", "-lpfng_b200", f"-L{CUDA / 'lib64'}", "-lcudart",
               f"-Wl,-rpath,$ORIGIN/{rpath}"]
        subprocess.run(cmd, check=True)
    print(f"built {out}")


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--reference", required=True, type=pathlib.Path, help="the reference checkout (read only)")
    ap.add_argument("--out", type=pathlib.Path, default=HERE / "_build" / "pfng-bench")
    ap.add_argument("--cxx", default="g++")
    args = ap.parse_args()
    if not (args.reference / "bench" / "main.cpp").exists():
        raise SystemExit(f"{args.reference} is not a reference checkout")
    build(args.reference, args.out, args.cxx)
    return 0


if __name__ == "__main__":
    sys.exit(main())
