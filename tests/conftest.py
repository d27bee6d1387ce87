import ctypes
import glob
import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
sys.path.insert(0, os.path.join(REPO, "kv-compact_b200", "python"))

from kvc_b200 import LIB_PATH, ORACLE_PATH, REF_PATH, abi  # noqa: E402

GOLDEN_DIR = os.path.join(REPO, "tests", "golden", "cases")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def oracle():
    """The C restatement (test infrastructure), bound with its oracle_ prefix."""
    if not os.path.exists(ORACLE_PATH):
        pytest.fail("oracle/liboracle.so missing: run `make -C oracle oracle`")
    lib = ctypes.CDLL(ORACLE_PATH, mode=ctypes.RTLD_LOCAL)
    fns = abi.bind(lib, prefix="oracle_")
    lib.oracle_select_only.restype = None
    lib.oracle_select_only.argtypes = [ctypes.c_int]
    fns["_lib"] = lib
    return fns


@pytest.fixture(scope="session")
def reflib():
    """The reference library compiled from source (oracle/_ref), if present."""
    if not os.path.exists(REF_PATH):
        pytest.skip("oracle/_ref/libkv-compact.so not built here")
    lib = ctypes.CDLL(REF_PATH, mode=ctypes.RTLD_LOCAL)
    return abi.bind(lib)


@pytest.fixture(scope="session")
def kvc():
    """libkvc.so bound through the drop-in ABI."""
    if not os.path.exists(LIB_PATH):
        pytest.fail("kv-compact_b200/lib/libkvc.so missing: run `make -C kv-compact_b200`")
    from kvc_b200 import lib as kvclib
    return kvclib.load()


def load_case(path):
    z = np.load(path)
    d = {k: z[k] for k in z.files}
    d["meta"] = json.loads(str(d["meta"]))
    for k in ("K", "V", "Q"):
        if k in d and d[k].dtype == np.float16:
            d[k] = np.ascontiguousarray(d[k].astype(np.float32))
    return d


def golden_cases(kind=None):
    out = []
    for p in sorted(glob.glob(os.path.join(GOLDEN_DIR, "*.npz"))):
        name = os.path.basename(p)[:-4]
        if kind is None or load_case(p)["meta"]["kind"] == kind:
            out.append(name)
    return out


def golden_path(name):
    return os.path.join(GOLDEN_DIR, name + ".npz")
