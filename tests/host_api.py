"""Builds tests/cpp/host_api_driver.cpp: a caller of the C++ drop-in API (host/include)
linked to the in-tree libqwen_cuda.so, as a maintainer's main.cpp would be."""
import os
import subprocess
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "qwen3.5-cpu-cpp_b200")
SRC = os.path.join(ROOT, "tests", "cpp", "host_api_driver.cpp")
_BIN = None


def driver():
    global _BIN
    if _BIN is None:
        out = os.path.join(tempfile.mkdtemp(prefix="qwc_host_api_"), "host_api_driver")
        subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(PKG, "host", "include"),
                        "-I", os.path.join(ROOT, "include"), SRC, "-L", PKG, "-lqwen_cuda",
                        f"-Wl,-rpath,{PKG}", "-o", out], check=True)
        _BIN = out
    return _BIN


def run(*args, timeout=600):
    return subprocess.run([driver()] + [str(a) for a in args], capture_output=True, text=True, timeout=timeout)


def read_st(path):
    """Parses the `st` command's output file."""
    b = open(path, "rb").read()
    o = 0

    def take(dt, n=1):
        nonlocal o
        a = np.frombuffer(b, dt, n, o)
        o += a.nbytes
        return a

    r = {"view_numel": int(take(np.int64)[0]), "view_kind": int(take(np.int32)[0])}
    n = int(take(np.int64)[0])
    r["f32_numel"] = n
    r["cached"] = bool(take(np.int32)[0])
    r["f32"] = take(np.float32, n) if r["cached"] else None
    r["row_ok"] = bool(take(np.int32)[0])
    w = int(take(np.int64)[0])
    r["row"] = take(np.float32, w) if r["row_ok"] else None
    r["oob_refused"] = bool(take(np.int32)[0])
    r["missing_refused"] = bool(take(np.int32)[0])
    return r
