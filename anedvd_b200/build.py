"""Build libcuq.so (the C-ABI CUDA library) in-tree with nvcc for sm_100a.

    python -m anedvd_b200.build        # or anedvd_b200.build.build()

Every source is compiled with `-gencode arch=compute_100a,code=sm_100a` and
linked into one shared library next to this file, so it travels with the
repository to a GPU box.  No JIT cache is involved.
"""
import os
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libcuq.so")
OBJ_DIR = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
         "-Xptxas", "-O3"]


def sources():
    out = []
    for f in sorted(os.listdir(CSRC)):
        if f.endswith((".cu", ".cpp")):
            out.append(os.path.join(CSRC, f))
    return out


def _headers_mtime():
    m = 0.0
    for d in (CSRC, os.path.join(os.path.dirname(HERE), "include")):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh")):
                m = max(m, os.path.getmtime(os.path.join(d, f)))
    return m


def build(force=False, verbose=False, jobs=None):
    os.makedirs(OBJ_DIR, exist_ok=True)
    hdr = _headers_mtime()
    objs, procs = [], []
    for src in sources():
        obj = os.path.join(OBJ_DIR, os.path.basename(src) + ".o")
        objs.append(obj)
        if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr):
            continue
        cmd = [NVCC] + ARCH + FLAGS + ["-c", src, "-o", obj]
        if src.endswith(".cpp"):
            cmd = [NVCC, "-x", "cu"] + ARCH + FLAGS + ["-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        if len(procs) >= (jobs or os.cpu_count() or 4):
            _drain(procs)
    _drain(procs)
    if force or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs
        r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
        if r.returncode:
            raise RuntimeError("link failed:\n" + r.stdout)
    return LIB


def _drain(procs):
    errs = []
    while procs:
        src, p = procs.pop(0)
        out, _ = p.communicate()
        if p.returncode:
            errs.append("%s:\n%s" % (src, out.decode(errors="replace")))
        elif out and b"warning" in out:
            sys.stderr.write(out.decode(errors="replace"))
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))


if __name__ == "__main__":
    t = time.time()
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
    print("built in %.1fs" % (time.time() - t))
