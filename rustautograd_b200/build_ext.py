"""Builds the native parts in-tree, incrementally.

* ``rustautograd_b200/lib/librgc_b200.so`` — the C-ABI CUDA device (``include/rgc.h``): kernels for
  sm_100a, plan lowering, run loop, NCCL data parallelism.
* ``rustautograd_b200/_rg*.so`` — the ``_rg`` Python module over that device.
* ``oracle/_build/_rg_oracle*.so`` — the CPU oracle module (test infrastructure only).

Every object is rebuilt only when one of its sources or headers is newer than it.
"""
import concurrent.futures as cf
import glob
import os
import subprocess
import sys
import sysconfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "rustautograd_b200")
HOST = os.path.join(PKG, "csrc", "host")
CUDA_DIR = os.path.join(PKG, "csrc", "cuda")
ORACLE = os.path.join(ROOT, "oracle")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

HOST_SOURCES = ["graph.cpp", "plan.cpp", "optimize.cpp", "egraph.cpp", "autodiff.cpp", "run.cpp", "validate.cpp", "blob.cpp", "rowchain.cpp"]


def _ext_suffix():
    return sysconfig.get_config_var("EXT_SUFFIX")


def _py_includes():
    import pybind11
    return ["-I" + sysconfig.get_paths()["include"], "-I" + pybind11.get_include()]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _headers():
    hs = glob.glob(os.path.join(HOST, "*.h")) + glob.glob(os.path.join(CUDA_DIR, "*.h")) + glob.glob(os.path.join(CUDA_DIR, "*.cuh"))
    hs += glob.glob(os.path.join(ORACLE, "*.h")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    return hs


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


CXXFLAGS = ["-O3", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wno-sign-compare", "-Wno-unused-function",
            "-ffp-contract=off", "-fno-math-errno"]


def _compile_all(jobs):
    """jobs: list of (target, deps, cmd). Runs the stale ones in parallel."""
    todo = [(t, c) for t, d, c in jobs if _stale(t, d)]
    if not todo:
        return
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        futs = [ex.submit(_run, c) for _, c in todo]
        for f in futs:
            f.result()


def build_oracle():
    """The CPU oracle module: host engine + CPU interpreter + pybind module (test infrastructure)."""
    out_dir = os.path.join(ORACLE, "_build")
    os.makedirs(out_dir, exist_ok=True)
    hdrs = _headers()
    jobs, objs = [], []
    srcs = [(os.path.join(HOST, s), []) for s in HOST_SOURCES]
    srcs.append((os.path.join(HOST, "pymod.cpp"), ["-DRG_MODULE_NAME=_rg_oracle"] + _py_includes()))
    srcs.append((os.path.join(ORACLE, "interp.cpp"), []))
    srcs.append((os.path.join(ORACLE, "module.cpp"), _py_includes()))
    for src, extra in srcs:
        obj = os.path.join(out_dir, os.path.basename(src) + ".o")
        jobs.append((obj, [src] + hdrs, ["g++"] + CXXFLAGS + extra + ["-c", src, "-o", obj]))
        objs.append(obj)
    _compile_all(jobs)
    target = os.path.join(out_dir, "_rg_oracle" + _ext_suffix())
    if _stale(target, objs):
        _run(["g++", "-shared", "-o", target] + objs + ["-lpthread"])
    return target


def _cuda_sources():
    return sorted(glob.glob(os.path.join(CUDA_DIR, "*.cu"))) + sorted(glob.glob(os.path.join(CUDA_DIR, "*.cpp")))


def build_device():
    """librgc_b200.so: the C-ABI CUDA device (host plan structures + kernels), built for sm_100a."""
    out_dir = os.path.join(PKG, "_build")
    lib_dir = os.path.join(PKG, "lib")
    os.makedirs(out_dir, exist_ok=True)
    os.makedirs(lib_dir, exist_ok=True)
    hdrs = _headers()
    jobs, objs = [], []
    inc = ["-I" + os.path.join(ROOT, "include"), "-I" + HOST, "-I" + CUDA_DIR, "-I" + os.path.join(CUDA_HOME, "include")]
    for s in HOST_SOURCES:
        src = os.path.join(HOST, s)
        obj = os.path.join(out_dir, "dev_" + s + ".o")
        jobs.append((obj, [src] + hdrs, ["g++"] + CXXFLAGS + inc + ["-c", src, "-o", obj]))
        objs.append(obj)
    for src in _cuda_sources():
        obj = os.path.join(out_dir, "dev_" + os.path.basename(src) + ".o")
        if src.endswith(".cu"):
            cmd = [NVCC] + ARCH + ["-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                                   "-fmad=false", "-prec-div=true", "-prec-sqrt=true"] + inc + ["-c", src, "-o", obj]
        else:
            cmd = ["g++"] + CXXFLAGS + inc + ["-c", src, "-o", obj]
        jobs.append((obj, [src] + hdrs, cmd))
        objs.append(obj)
    _compile_all(jobs)
    target = os.path.join(lib_dir, "librgc_b200.so")
    if _stale(target, objs):
        _run(["g++", "-shared", "-o", target] + objs + ["-L" + os.path.join(CUDA_HOME, "lib64"), "-lcudart", "-lnvrtc", "-ldl", "-lpthread",
                                                         "-Wl,-rpath," + os.path.join(CUDA_HOME, "lib64")])
    return target


def build_module():
    """The product `_rg` module: host engine + pybind module, executing through librgc_b200.so."""
    out_dir = os.path.join(PKG, "_build")
    os.makedirs(out_dir, exist_ok=True)
    hdrs = _headers()
    jobs, objs = [], []
    inc = ["-I" + os.path.join(ROOT, "include"), "-I" + HOST]
    for s in HOST_SOURCES:
        src = os.path.join(HOST, s)
        obj = os.path.join(out_dir, "mod_" + s + ".o")
        jobs.append((obj, [src] + hdrs, ["g++"] + CXXFLAGS + inc + ["-c", src, "-o", obj]))
        objs.append(obj)
    for src, extra in [(os.path.join(HOST, "pymod.cpp"), ["-DRG_MODULE_NAME=_rg"] + _py_includes()),
                       (os.path.join(PKG, "csrc", "cuda_client.cpp"), _py_includes())]:
        obj = os.path.join(out_dir, "mod_" + os.path.basename(src) + ".o")
        jobs.append((obj, [src] + hdrs, ["g++"] + CXXFLAGS + inc + extra + ["-c", src, "-o", obj]))
        objs.append(obj)
    _compile_all(jobs)
    target = os.path.join(PKG, "_rg" + _ext_suffix())
    lib_dir = os.path.join(PKG, "lib")
    if _stale(target, objs + [os.path.join(lib_dir, "librgc_b200.so")]):
        _run(["g++", "-shared", "-o", target] + objs + ["-L" + lib_dir, "-lrgc_b200", "-Wl,-rpath,$ORIGIN/lib", "-lpthread"])
    return target


def build_all():
    build_oracle()
    build_device()
    build_module()


if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else "all"
    {"oracle": build_oracle, "device": build_device, "module": build_module, "all": build_all}[what]()
    print("built", what)
