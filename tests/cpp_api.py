"""Builds tests/cpp/api_decode.cpp against libvxb (shared by the CPU and GPU tests)."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "voxcpm-inference_b200")


def build_api_decode(out_dir: str) -> str:
    exe = os.path.join(out_dir, "api_decode")
    subprocess.run(["g++", "-std=c++17", "-O2", "-I", os.path.join(PKG, "include"),
                    os.path.join(ROOT, "tests", "cpp", "api_decode.cpp"), "-L", os.path.join(PKG, "lib"), "-lvxb",
                    "-Wl,-rpath," + os.path.join(PKG, "lib"), "-o", exe], check=True)
    return exe
