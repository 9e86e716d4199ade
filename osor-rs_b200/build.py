"""Builds libosor_b200.so (sm_100a) in-tree with nvcc.

Usage: python osor-rs_b200/build.py [--clean]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "osor_b200")
LIB = os.path.join(OUT_DIR, "libosor_b200.so")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-rdc=true",
         "-I" + INCLUDE, "-I" + CSRC]
SOURCES = ["conv_tc.cu", "conv_tc2.cu", "conv_tcn.cu", "attn_fa.cu", "groupnorm.cu", "ops.cu", "vae.cu", "capi.cu", "profile.cu", "gn_noalloc.cu", "noise.cu", "pipeline.cu", "unet.cu", "unet_model.cu", "conv_out.cu", "attn_pair.cu", "attn_heads.cu", "peer.cu", "vae_band.cu"]


def _compile(src: str) -> str:
    obj = os.path.join(BUILD, src.replace(".cu", ".o"))
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(INCLUDE, "osor_b200.h")]
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
    subprocess.run(cmd, check=True)
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(_compile, SOURCES))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        # nvcc performs the device link of the relocatable objects.
        cmd = [NVCC, *ARCH, "-shared", "-rdc=true", "-Xcompiler", "-fPIC", "-o", LIB, *objs,
               "-cudart", "static", "-ldl", "-lrt", "-lpthread"]
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    if "--clean" in sys.argv:
        shutil.rmtree(BUILD, ignore_errors=True)
        if os.path.exists(LIB):
            os.remove(LIB)
    print(build())
