"""Builds the renderer in-tree for sm_100a.

* ``libvi_b200.so``  -- the CUDA kernels and the C ABI (include/volume_integration_b200.h),
  compiled with nvcc ``-gencode arch=compute_100a,code=sm_100a -O3 -lineinfo``;
* ``_C*.so``         -- the torch binding with the reference's Python signatures,
  linked against libvi_b200.so with an $ORIGIN rpath.

Both land in ``volume_integration/``; objects go to ``_build/``.  Rebuilds only
what is older than its sources.
"""
import concurrent.futures as cf
import glob
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
PKG = os.path.join(HERE, "volume_integration")
OBJ = os.path.join(HERE, "_build", "obj")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libvi_b200.so")
SOURCES = ["vi_sort.cu", "vi_binning.cu", "vi_features.cu", "vi_render.cu", "vi_backward.cu", "vi_api.cu",
           "vi_sort_noalloc.cu", "vi_gaussians.cu", "vi_table.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _host_compilers():
    """The distribution's gcc/g++, the toolchain torch's own C++ runtime matches.
    A wrapper that points g++ at another GCC's support files (crt objects, libgcc)
    builds an extension whose C++ exceptions crash while they are formatted, so
    the system compilers are preferred when they exist."""
    cc, cxx = "/usr/bin/gcc", "/usr/bin/g++"
    return (cc, cxx) if os.path.exists(cc) and os.path.exists(cxx) else (None, None)


_CC, _CXX = _host_compilers()
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I" + INCLUDE] + \
    (["-ccbin", _CXX] if _CXX else [])


def _nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.sep not in c or os.path.exists(c)):
            return c
    return "nvcc"


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, obj):
    cmd = [_nvcc()] + NVCC_FLAGS + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s%s" % (src, r.stdout, r.stderr))
    return obj


def build_lib(force=False, jobs=6):
    os.makedirs(OBJ, exist_ok=True)
    hdrs = _headers()
    work = []
    objs = []
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(OBJ, s.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            work.append((src, obj))
    if work:
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            for f in [ex.submit(_compile, s, o) for s, o in work]:
                f.result()
    if force or work or _stale(LIB, objs):
        cmd = [_nvcc()] + ARCH + (["-ccbin", _CXX] if _CXX else []) + ["-shared", "-o", LIB] + objs
        subprocess.run(cmd, check=True)
    return LIB


def _ext_path():
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return os.path.join(PKG, "_C" + suffix)


def build_ext(force=False):
    target = _ext_path()
    deps = [os.path.join(CSRC, "ext.cpp"), os.path.join(INCLUDE, "volume_integration_b200.h"), LIB]
    if not force and not _stale(target, deps):
        return target
    script = r"""
import sys
from setuptools import setup
from torch.utils.cpp_extension import CUDAExtension, BuildExtension
setup(name="volume_integration_b200_ext",
      ext_modules=[CUDAExtension("volume_integration._C", ["csrc/ext.cpp"],
                                 include_dirs=[%r], library_dirs=["volume_integration"],
                                 libraries=["vi_b200"],
                                 extra_compile_args={"cxx": ["-O2", "-std=c++17"]},
                                 extra_link_args=["-Wl,-rpath,$ORIGIN"])],
      cmdclass={"build_ext": BuildExtension},
      script_args=["-q", "build_ext", "--inplace", "--build-temp", "_build/ext"])
""" % INCLUDE
    env = dict(os.environ)
    if _CXX:
        env["CC"], env["CXX"] = _CC, _CXX
    env.setdefault("MAX_JOBS", "4")
    env["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    r = subprocess.run([sys.executable, "-c", script], cwd=HERE, capture_output=True, text=True, env=env)
    if r.returncode != 0:
        raise RuntimeError("torch binding build failed:\n%s%s" % (r.stdout[-4000:], r.stderr[-4000:]))
    return target


def build(force=False):
    build_lib(force)
    build_ext(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(LIB)
    print(_ext_path())
