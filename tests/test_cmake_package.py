"""The CMake install package (CMakeLists.txt), no GPU needed.

The sgBLAS install package is `find_package(sgblas 0.1 CONFIG REQUIRED)` plus
the `sgblas::sgblas` target (reference CMakeLists.txt: install(EXPORT
sgblasTargets NAMESPACE sgblas::), cmake/sgblasConfig.cmake.in, and its
cmake/install-consumer project). This test configures and builds the
repository with CMake, installs it into a fresh prefix, and builds and runs
a consumer project (tests/cmake_consumer) that only knows the package name.

The CMake build tree is kept in sgblas_b200/_build/cmake, so only the first
run compiles the kernels (about a minute and a half on 8 cores).
"""
import os
import pathlib
import shutil
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
BUILD = ROOT / "sgblas_b200" / "_build" / "cmake"
CONSUMER = ROOT / "tests" / "cmake_consumer"

NVCC_FOUND = shutil.which("nvcc") is not None or os.path.exists("/usr/local/cuda/bin/nvcc")
pytestmark = pytest.mark.skipif(shutil.which("cmake") is None or not NVCC_FOUND,
                                reason="cmake and nvcc are needed")


def run(cmd, **kw):
    res = subprocess.run([str(c) for c in cmd], capture_output=True, text=True, **kw)
    return res


def exported(lib):
    out = run(["nm", "-D", "--defined-only", lib]).stdout
    return sorted(line.split()[-1] for line in out.splitlines() if " T " in line)


@pytest.fixture(scope="module")
def prefix(tmp_path_factory):
    env = dict(os.environ)
    if shutil.which("nvcc") is None:
        env["CUDACXX"] = "/usr/local/cuda/bin/nvcc"
    cfg = run(["cmake", "-S", ROOT, "-B", BUILD, "-DCMAKE_BUILD_TYPE=Release"], env=env)
    assert cfg.returncode == 0, cfg.stdout + cfg.stderr
    bld = run(["cmake", "--build", BUILD, "-j", str(min(8, os.cpu_count() or 1))], env=env,
              timeout=1800)
    assert bld.returncode == 0, bld.stdout[-4000:] + bld.stderr[-4000:]
    dest = tmp_path_factory.mktemp("sgblas_prefix")
    inst = run(["cmake", "--install", BUILD, "--prefix", dest])
    assert inst.returncode == 0, inst.stdout + inst.stderr
    return dest


def test_install_layout(prefix):
    libdir = next(p for p in (prefix / "lib", prefix / "lib64") if p.exists())
    for h in ("sgblas.h", "sgblas_ext.h", "sgblas_mg.h"):
        installed = (prefix / "include" / "sgblas" / h).read_bytes()
        assert installed == (ROOT / "include" / "sgblas" / h).read_bytes(), h
    for f in ("sgblasConfig.cmake", "sgblasConfigVersion.cmake", "sgblasTargets.cmake"):
        assert (libdir / "cmake" / "sgblas" / f).exists(), f
    real = libdir / "libsgblas.so.0.1.0"
    assert real.exists() and (libdir / "libsgblas.so").resolve() == real.resolve()
    # The CMake build exports exactly the C API that the Python build exports.
    in_tree = ROOT / "sgblas_b200" / "lib" / "libsgblas.so"
    names = exported(real)
    assert "sgblasSgemm" in names and all(n.startswith("sgblas") for n in names), names
    if in_tree.exists():
        assert names == exported(in_tree)
    needed = run(["readelf", "-d", real]).stdout
    assert "libcudart" not in needed and "libsgblas.so.0" in needed, needed


def test_consumer_finds_links_and_runs(prefix, tmp_path):
    build = tmp_path / "consumer"
    cfg = run(["cmake", "-S", CONSUMER, "-B", build, f"-DCMAKE_PREFIX_PATH={prefix}"])
    assert cfg.returncode == 0, cfg.stdout + cfg.stderr
    bld = run(["cmake", "--build", build])
    assert bld.returncode == 0, bld.stdout + bld.stderr
    exe = build / "sgblas_cmake_consumer"
    libs = run(["ldd", exe]).stdout
    assert str(prefix) in libs, libs   # the installed library, through the target's rpath
    res = run([exe], timeout=60)
    assert res.returncode == 0 and "invalid value" in res.stdout.lower(), (res.returncode,
                                                                          res.stdout, res.stderr)


def test_version_compatibility(prefix, tmp_path):
    """0.x packages accept requests for the same minor version only."""
    ok = run(["cmake", "-S", CONSUMER, "-B", tmp_path / "same", f"-DCMAKE_PREFIX_PATH={prefix}",
              "-DSGBLAS_WANTED_VERSION=0.1.0"])
    assert ok.returncode == 0, ok.stdout + ok.stderr
    newer = run(["cmake", "-S", CONSUMER, "-B", tmp_path / "newer",
                 f"-DCMAKE_PREFIX_PATH={prefix}", "-DSGBLAS_WANTED_VERSION=0.2"])
    assert newer.returncode != 0
    assert "sgblas" in (newer.stdout + newer.stderr)
