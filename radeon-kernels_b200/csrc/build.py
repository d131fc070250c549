"""Build the sm_100a kernel library, its PyTorch bindings and the built-in kernel pack.

Outputs (all git-ignored binaries, built in-tree so they travel with the source tree):

* ``radeon_kernels/_lib/librk_kernels.so`` -- every CUDA kernel behind the C ABI of
  ``include/rk_kernels.h`` (static CUDA runtime, no PyTorch dependency);
* ``radeon_kernels/_lib/_rk_ext<EXT_SUFFIX>`` -- PyTorch binding used by the built-in
  ``cuda`` provider (links ``librk_kernels.so`` through ``$ORIGIN``);
* ``radeon_kernels/_packs/rk-sm100a/lib/rk_sm100a.so`` -- the same binding with the
  kernels linked in, published as the ``python_extension`` artifact of the built-in
  sm_100a kernel pack; ``manifest.json`` beside it records its SHA-256, and the sm_100a
  entries of ``dispatch/*.json`` are refreshed to the same digest.

Incremental: a step reruns only when one of its inputs is newer than its output.
Usage: ``python radeon-kernels_b200/csrc/build.py [--force] [--jobs N]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG_ROOT = CSRC.parent  # radeon-kernels_b200/
PACKAGE = PKG_ROOT / "radeon_kernels"
REPO = PKG_ROOT.parent
INCLUDE = REPO / "include"
BUILD = PKG_ROOT / "_build"
LIB_DIR = PACKAGE / "_lib"
PACK_DIR = PACKAGE / "_packs" / "rk-sm100a"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH_FLAGS,
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]
KERNEL_SOURCES = ["rk_abi.cu", "peer.cu", "gemm_tcgen05.cu", "gemm_tcgen05_2sm.cu", "gemm_simt.cu", "gemv.cu", "gemv_tcgen05.cu", "gather.cu", "llm_ops.cu", "llm_ops_backward.cu", "paged_attention.cu", "paged_attention_tc.cu", "sdpa_tcgen05.cu"]
HEADERS = sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "rk_kernels.h"]

REPRODUCIBLE_LINK = ["-Wl,--strip-all", "-Wl,--build-id=none"]
EXT_SUFFIX = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
LIBRARY = LIB_DIR / "librk_kernels.so"
BUILTIN_EXT = LIB_DIR / f"_rk_ext{EXT_SUFFIX}"
PACK_EXT = PACK_DIR / "lib" / "rk_sm100a.so"


def _stale(output: Path, inputs: list[Path], force: bool) -> bool:
    if force or not output.exists():
        return True
    stamp = output.stat().st_mtime
    return any(path.stat().st_mtime > stamp for path in inputs)


def _run(cmd: list[str]) -> None:
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        sys.stderr.write(result.stdout + result.stderr)
        raise RuntimeError(f"command failed ({result.returncode}): {' '.join(cmd[:6])} ...")


def _compile_cuda(source: Path, force: bool) -> Path:
    obj = BUILD / "obj" / (source.stem + ".o")
    if _stale(obj, [source, *HEADERS], force):
        obj.parent.mkdir(parents=True, exist_ok=True)
        # A fixed seed keeps the host compiler's generated names the same from build to build.
        _run([NVCC, *NVCC_FLAGS, f"-Xcompiler=-frandom-seed={source.stem}", "-c", str(source), "-o", str(obj)])
    return obj


def _torch_flags() -> tuple[list[str], list[str]]:
    import torch
    from torch.utils import cpp_extension

    includes = [f"-I{path}" for path in cpp_extension.include_paths(device_type="cuda")]
    includes.append(f"-I{sysconfig.get_paths()['include']}")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cflags = [
        "-O2",
        "-std=c++17",
        "-fPIC",
        "-fvisibility=hidden",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        *includes,
        f"-I{INCLUDE}",
    ]
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    ldflags = [
        f"-L{torch_lib}",
        "-lc10",
        "-lc10_cuda",
        "-ltorch",
        "-ltorch_cpu",
        "-ltorch_python",
    ]
    return cflags, ldflags


def _compile_binding(name: str, cflags: list[str], force: bool) -> Path:
    source = CSRC / "torch_ext.cpp"
    obj = BUILD / "obj" / f"torch_ext_{name}.o"
    if _stale(obj, [source, INCLUDE / "rk_kernels.h"], force):
        obj.parent.mkdir(parents=True, exist_ok=True)
        _run(["g++", *cflags, f"-frandom-seed=torch_ext_{name}", f"-DTORCH_EXTENSION_NAME={name}", "-c", str(source),
              "-o", str(obj)])
    return obj


def build(*, force: bool = False, jobs: int | None = None) -> dict[str, Path]:
    """Build every artifact; returns their paths."""

    BUILD.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    (PACK_DIR / "lib").mkdir(parents=True, exist_ok=True)
    cflags, ldflags = _torch_flags()
    workers = jobs or min(8, os.cpu_count() or 2)
    with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
        kernel_jobs = [pool.submit(_compile_cuda, CSRC / src, force) for src in KERNEL_SOURCES]
        binding_jobs = {
            name: pool.submit(_compile_binding, name, cflags, force) for name in ("_rk_ext", "rk_sm100a")
        }
        objects = [job.result() for job in kernel_jobs]
        bindings = {name: job.result() for name, job in binding_jobs.items()}

    # Reproducible links: nvcc records its per-process temporary file names in the host
    # symbol table, so the libraries are linked without .symtab (--strip-all; the exported
    # .dynsym and the kernels' line information in the device code stay) and without a
    # build id -- the same sources and toolchain give byte-identical binaries, so the pack
    # digests in the tracked manifests change only when the code does.
    if _stale(LIBRARY, objects, force):
        _run([NVCC, *ARCH_FLAGS, "-shared", "-o", str(LIBRARY), *map(str, objects), "-cudart", "static",
              "-Xlinker", "--strip-all,--build-id=none"])

    cudart = ["-L" + str(CUDA_HOME / "lib64"), "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
    if _stale(BUILTIN_EXT, [bindings["_rk_ext"], LIBRARY], force):
        _run(
            [
                "g++",
                "-shared",
                "-o",
                str(BUILTIN_EXT),
                str(bindings["_rk_ext"]),
                f"-L{LIB_DIR}",
                "-lrk_kernels",
                "-Wl,-rpath,$ORIGIN",
                *ldflags,
                *REPRODUCIBLE_LINK,
            ]
        )
    pack_built = False
    if _stale(PACK_EXT, [bindings["rk_sm100a"], *objects], force):
        _run(["g++", "-shared", "-o", str(PACK_EXT), str(bindings["rk_sm100a"]), *map(str, objects), *ldflags, *cudart,
              *REPRODUCIBLE_LINK])
        pack_built = True

    sys.path.insert(0, str(PKG_ROOT))
    from radeon_kernels.runtime.publish import load_private_key, publish_builtin_pack, sign_manifest
    from radeon_kernels.runtime.signing import builtin_trusted_keyring

    publish_builtin_pack(PACK_DIR, PACK_EXT, refresh_dispatch=False, rewrite=pack_built)
    key_file = release_key_file()
    key, key_id = load_private_key(key_file) if key_file is not None else (None, None)
    sign_manifest(PACK_DIR, key, key_id, builtin_trusted_keyring())
    return {"library": LIBRARY, "builtin_extension": BUILTIN_EXT, "pack_extension": PACK_EXT}


def release_key_file() -> Path | None:
    """The release signing key: $RADEON_KERNELS_RELEASE_KEY, else the one ``<key_id>.pem`` in
    the repository's git-ignored ``.release-key/`` directory, else none (unsigned build)."""

    named = os.environ.get("RADEON_KERNELS_RELEASE_KEY")
    if named:
        return Path(named)
    found = sorted((REPO / ".release-key").glob("*.pem"))
    return found[-1] if found else None


def clean() -> None:
    shutil.rmtree(BUILD, ignore_errors=True)


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true", help="rebuild everything")
    parser.add_argument("--jobs", type=int, default=None)
    args = parser.parse_args(argv)
    for key, path in build(force=args.force, jobs=args.jobs).items():
        print(f"{key}: {path.relative_to(REPO)}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
