"""Build the two native artefacts of the engine, in-tree, for sm_100a.

  fable_attn/libfable_attn.so   CUDA kernels + the extern "C" API of include/fable_attn.h
                                (nvcc, -gencode arch=compute_100a,code=sm_100a, static cudart)
  fable_attn/_C.<abi>.so        torch extension (pybind) that marshals tensors into the C-ABI
                                parameter blocks; links libfable_attn.so with rpath $ORIGIN

Objects are compiled in parallel and rebuilt only when a source or header is newer than the
artefact.  Usage: python build.py [--force] [--no-ext]
"""
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
PKG = os.path.join(HERE, "fable_attn")
INC = os.path.join(ROOT, "include")
OBJ = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           "--expt-relaxed-constexpr", "-I", INC, "-I", CSRC]

KERNEL_SOURCES = ["api.cu", "fwd_simt.cu", "fwd_sm100.cu", "bwd_simt.cu", "bwd_sm100.cu", "decode.cu", "decode_sm100.cu", "dropout.cu", "rotary.cu",
                  "decode_peer.cu"]
LIB = os.path.join(PKG, "libfable_attn.so")


def _headers():
    hs = [os.path.join(INC, f) for f in os.listdir(INC)]
    hs += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    return hs


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("command failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def build_lib(force=False, verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    hdrs = _headers()
    jobs = []
    objs = []
    for s in KERNEL_SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(OBJ, s + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            jobs.append([NVCC] + ARCH + NVFLAGS + ["-Xptxas", "-v", "-c", src, "-o", obj])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for out in ex.map(_run, jobs):
            if verbose:
                print(out)
    if force or jobs or _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", LIB] + objs)
    return LIB


def build_ext(force=False):
    import torch.utils.cpp_extension as ce
    suffix = sysconfig.get_config_var("EXT_SUFFIX")
    out = os.path.join(PKG, "_C" + suffix)
    src = os.path.join(CSRC, "dispatch.cpp")
    if not force and not _stale(out, [src, LIB] + _headers()):
        return out
    py_inc = sysconfig.get_paths()["include"]
    incs = ce.include_paths() + [py_inc, INC, CSRC, "/usr/local/cuda/include"]
    libdirs = ce.library_paths()
    import torch
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    cmd += [f"-I{i}" for i in incs]
    cmd += [src, "-o", out]
    cmd += [f"-L{d}" for d in libdirs] + [f"-Wl,-rpath,{d}" for d in libdirs]
    cmd += ["-L" + PKG, "-Wl,-rpath,$ORIGIN", "-l:libfable_attn.so",
            "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python"]
    _run(cmd)
    return out


def main(argv):
    force = "--force" in argv
    lib = build_lib(force=force, verbose="-v" in argv)
    print("built", lib)
    if "--no-ext" not in argv:
        print("built", build_ext(force=force))


if __name__ == "__main__":
    main(sys.argv[1:])
