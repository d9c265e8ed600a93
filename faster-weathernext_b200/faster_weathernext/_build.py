"""Builds libfwn_attn.so in-tree with nvcc for sm_100a (no JIT cache, no pip install).

    python -m faster_weathernext._build            # from faster-weathernext_b200/
"""

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(os.path.dirname(ROOT), "include")
LIB = os.path.join(PKG, "libfwn_attn.so")
SOURCES = ["fwn_attn.cu", "tiles.cu", "khop.cu", "norm.cu", "gnn.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr"]


def nvcc():
  path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
  if not os.path.exists(path):
    raise RuntimeError("nvcc not found; libfwn_attn.so cannot be built")
  return path


def _inputs():
  files = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".h"))]
  files += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
  return files


def up_to_date() -> bool:
  if not os.path.exists(LIB):
    return False
  t = os.path.getmtime(LIB)
  return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
  """Compile csrc/*.cu into faster_weathernext/libfwn_attn.so; returns its path."""
  if not force and up_to_date():
    return LIB
  out_dir = os.path.join(ROOT, "_build")
  os.makedirs(out_dir, exist_ok=True)
  objs = []
  for src in SOURCES:
    obj = os.path.join(out_dir, src.replace(".cu", ".o"))
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", INCLUDE, "-c", os.path.join(CSRC, src), "-o", obj]
    if verbose:
      cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    objs.append(obj)
  tmp = LIB + ".tmp"
  subprocess.run([nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-lcudart_static", "-ldl",
                  "-lrt", "-lpthread"], check=True)
  os.replace(tmp, LIB)
  return LIB


if __name__ == "__main__":
  print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
