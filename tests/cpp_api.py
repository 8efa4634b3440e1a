"""Builds the C++ API callers in tests/cpp/ against libvxb (shared by the CPU and GPU tests)."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "voxcpm-inference_b200")


def build_caller(out_dir: str, name: str) -> str:
    exe = os.path.join(out_dir, name)
    subprocess.run(["g++", "-std=c++17", "-O2", "-I", os.path.join(PKG, "include"),
                    os.path.join(ROOT, "tests", "cpp", name + ".cpp"), "-L", os.path.join(PKG, "lib"), "-lvxb",
                    "-Wl,-rpath," + os.path.join(PKG, "lib"), "-o", exe], check=True)
    return exe


def build_api_decode(out_dir: str) -> str:
    return build_caller(out_dir, "api_decode")


def build_api_encode(out_dir: str) -> str:
    return build_caller(out_dir, "api_encode")
