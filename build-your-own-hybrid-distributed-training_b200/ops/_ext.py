"""Build and load the native extension ``hybrid_training.ops._C``.

Every CUDA source under ``ops/csrc`` is compiled for ``sm_100a`` only
(``-gencode arch=compute_100a,code=sm_100a``) into one in-tree shared object,
so it travels with the source tree and is found without a JIT cache.  The
extension does not link ``libcuda``: the driver entry points it needs (tensor
map encoding, multicast objects) are fetched through the runtime at first use,
so the module imports on machines without a GPU driver.

On a CUDA tensor every op in :mod:`hybrid_training.ops` runs the native kernel;
if the extension cannot be loaded the op raises :class:`KernelError` instead of
falling back to a PyTorch implementation.
"""

from __future__ import annotations

import glob
import importlib.util
import os
import sys
import sysconfig
from pathlib import Path
from types import ModuleType

from ..errors import KernelError, format_error

__all__ = ["ARCH_FLAGS", "build_checked_extension", "build_extension", "checked_extension", "checked_extension_path",
           "extension", "extension_path", "has_extension"]

_HERE = Path(__file__).resolve().parent
_CSRC = _HERE / "csrc"
_BUILD_DIR = _HERE / "_build"
_NAME = "_C"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]

_module: ModuleType | None = None
_load_error: str | None = None


def extension_path() -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return _HERE / f"{_NAME}{suffix}"


def _sources() -> list[str]:
    return sorted(glob.glob(str(_CSRC / "*.cu")) + glob.glob(str(_CSRC / "*.cpp")))


def _libstdcxx_link_flags() -> list[str]:
    """Link the C++ runtime that this Python process already uses, as a shared library.

    When the toolchain's ``libstdc++.so`` link is missing, ``g++ -shared`` silently falls back to
    ``libstdc++.a``.  A second, static copy of the C++ runtime inside the extension then formats
    error messages through locale data that the process's own copy initialised, and crashes.  The
    mapped ``libstdc++.so.6`` of this process (torch loads it) is passed to the linker by path.
    """
    import torch  # noqa: F401  (maps the C++ runtime)

    try:
        with open("/proc/self/maps") as maps:
            for line in maps:
                path = line.split()[-1]
                if "libstdc++.so" in path and os.path.exists(path):
                    return [path]
    except OSError:
        pass
    return []


def build_extension(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile all sources (ninja, incremental) and place ``_C*.so`` next to this file."""
    from torch.utils import cpp_extension

    _BUILD_DIR.mkdir(exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(jobs or max(os.cpu_count() or 1, 1)))
    # Build into the scratch folder, then move the product in-tree.
    cuda_flags = [*ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "--use_fast_math", "-Xptxas=-v" if verbose else "-Xptxas=-O3",
                  "--expt-relaxed-constexpr", "-DNDEBUG", f"-I{_CSRC}"]
    cpp_extension.load(
        name=_NAME,
        sources=_sources(),
        build_directory=str(_BUILD_DIR),
        extra_cflags=["-O3", "-std=c++17", f"-I{_CSRC}"],
        extra_cuda_cflags=cuda_flags,
        extra_ldflags=_libstdcxx_link_flags(),
        verbose=verbose,
        is_python_module=True,
        with_cuda=True,
    )
    built = _BUILD_DIR / f"{_NAME}.so"
    target = extension_path()
    if built.exists():
        tmp = target.with_suffix(".tmp")
        tmp.write_bytes(built.read_bytes())
        tmp.replace(target)
    return target


_CHECKED_NAME = "_C_checked"
_checked_module: ModuleType | None = None


def checked_extension_path() -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return _HERE / f"{_CHECKED_NAME}{suffix}"


def build_checked_extension(verbose: bool = False) -> Path:
    """Compile the bounds-checked module (``csrc/checked``, ``-DHT_BOUNDS_CHECK``) next to the regular one."""
    from torch.utils import cpp_extension

    build_dir = _HERE / "_build_checked"
    build_dir.mkdir(exist_ok=True)
    cuda_flags = [*ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "--use_fast_math", "--expt-relaxed-constexpr", "-DNDEBUG",
                  f"-I{_CSRC}"]
    cpp_extension.load(name=_CHECKED_NAME, sources=[str(_CSRC / "checked" / "checked_ops.cu")], build_directory=str(build_dir),
                       extra_cflags=["-O3", "-std=c++17", f"-I{_CSRC}"], extra_cuda_cflags=cuda_flags,
                       extra_ldflags=_libstdcxx_link_flags(), verbose=verbose, is_python_module=True, with_cuda=True)
    built = build_dir / f"{_CHECKED_NAME}.so"
    target = checked_extension_path()
    if built.exists():
        tmp = target.with_suffix(".tmp")
        tmp.write_bytes(built.read_bytes())
        tmp.replace(target)
    return target


def checked_extension() -> ModuleType:
    """The bounds-checked module (built by :func:`build_checked_extension`); raises if it is missing."""
    global _checked_module
    if _checked_module is None:
        path = checked_extension_path()
        if not path.exists():
            raise KernelError(format_error("ops.checked_extension", "the bounds-checked module has not been built",
                                           expected=str(path), observed="missing",
                                           resolution="run hybrid_training.ops.build_checked_extension()"))
        import torch  # noqa: F401

        spec = importlib.util.spec_from_file_location(f"hybrid_training.ops.{_CHECKED_NAME}", path)
        assert spec is not None and spec.loader is not None
        module = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(module)
        _checked_module = module
    return _checked_module


def extension() -> ModuleType:
    """The loaded native module; raises :class:`KernelError` if it is unavailable."""
    global _module, _load_error
    if _module is not None:
        return _module
    if _load_error is None:
        path = extension_path()
        try:
            if not path.exists():
                raise FileNotFoundError(f"{path.name} has not been built")
            import torch  # noqa: F401  (the extension links against libtorch)

            spec = importlib.util.spec_from_file_location(f"hybrid_training.ops.{_NAME}", path)
            assert spec is not None and spec.loader is not None
            module = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(module)
            sys.modules[spec.name] = module
            _module = module
            return module
        except Exception as exc:  # pragma: no cover - depends on the build
            _load_error = f"{type(exc).__name__}: {exc}"
    raise KernelError(format_error("ops.extension", "the native sm_100a extension could not be loaded",
                                   expected=str(extension_path()), observed=_load_error,
                                   resolution="run `python -c 'import __graft_entry__ as g; g.build()'` "
                                              "(or hybrid_training.ops.build_extension()) on a machine with nvcc"))


def has_extension() -> bool:
    try:
        extension()
        return True
    except KernelError:
        return False
