"""Build the sm_100a shared library in-tree: synapse_b200/libsynapse_b200.so.

nvcc compiles every csrc/*.cu (CUDA kernels + the C ABI) and csrc/host/*.cpp
(the C++20 loader, planner and session) for sm_100a only. --fmad=false keeps
a*b+c as two roundings, the reference's -ffp-contract=off. First, gcc builds and
runs csrc/libm_expf_scan.c, which writes the device table of the inputs where
the host C library's expf rounds differently (_build/libm_expf_exc.inc).
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libsynapse_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_paths():
    try:
        import nvidia.nccl
        base = os.path.dirname(nvidia.nccl.__file__) if nvidia.nccl.__file__ else list(nvidia.nccl.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    except Exception:
        pass
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def libm_table(objdir, verbose=False):
    """The host C library's expf exceptions as a device table (csrc/libm_expf_scan.c), remade when missing or
    older than its sources; the device expf follows the host library on those inputs."""
    out = os.path.join(objdir, "libm_expf_exc.inc")
    srcs = [os.path.join(HERE, "csrc", "libm_expf_scan.c"), os.path.join(HERE, "csrc", "exp_table.h")]
    if os.path.exists(out) and all(os.path.getmtime(out) > os.path.getmtime(f) for f in srcs):
        return out
    exe = os.path.join(objdir, "libm_expf_scan")
    cmd = ["gcc", "-O2", "-ffp-contract=off", "-pthread", "-o", exe, srcs[0], "-lm"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    subprocess.run([exe, out + ".tmp"], check=True, stdout=None if verbose else subprocess.DEVNULL)
    os.replace(out + ".tmp", out)
    return out


def sources():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu"))) + \
        sorted(glob.glob(os.path.join(HERE, "csrc", "host", "*.cpp")))


def needs_build():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(HERE, "csrc", "*.cuh")) + glob.glob(os.path.join(HERE, "csrc", "*.h")) + \
        glob.glob(os.path.join(HERE, "csrc", "*.c")) + \
        glob.glob(os.path.join(HERE, "csrc", "host", "*.hpp")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    return any(os.path.getmtime(f) > t for f in deps)


def build(verbose=False, force=False):
    if not force and not needs_build():
        return LIB
    inc, libdir = nccl_paths()
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    libm_table(objdir, verbose)
    objs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        cmd = ["nvcc", *ARCH, "-O3", "-lineinfo", "--fmad=false", "-std=c++20", "-Xcompiler", "-fPIC",
               "-I", os.path.join(ROOT, "include"), "-I", objdir, "-I", inc, "-c", src, "-o", obj]
        if src.endswith(".cpp"):
            cmd = ["g++", "-O2", "-std=c++20", "-fPIC", "-Wall", "-I", os.path.join(ROOT, "include"),
                 "-I", inc, "-I", "/usr/local/cuda/include", "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(obj)
    link = ["nvcc", *ARCH, "-shared", "-o", LIB, *objs, "-L", libdir, "-lnccl", "-lcudart",
            "-Xlinker", "-rpath=" + libdir]
    if verbose:
        print(" ".join(link))
    subprocess.run(link, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
