"""Python host side of the B200 kv-compact library.

``abi``       ctypes mirror of the drop-in C ABI (include/kv-compact-api.h)
``lib``       loader for libkvc.so and wrappers over its entry points
``workloads`` seeded synthetic caches for the benchmark configurations
"""
import os

PKG_ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
REPO_ROOT = os.path.abspath(os.path.join(PKG_ROOT, ".."))
LIB_PATH = os.path.join(PKG_ROOT, "lib", "libkvc.so")
ORACLE_PATH = os.path.join(REPO_ROOT, "oracle", "liboracle.so")
REF_PATH = os.path.join(REPO_ROOT, "oracle", "_ref", "libkv-compact.so")
