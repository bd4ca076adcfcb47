"""Build the oracle (test infrastructure) and, where the reference tree is
present, the reference's own code into oracle/_ref/.

    python oracle/build_oracle.py [--force]

Outputs:
  oracle/liboracle.so            CPU restatement of the reference math (oracle.cpp)
  oracle/_ref/libref_sampler.so  the reference's sampler.h, compiled as is from
                                 the reference tree (CPU)
  oracle/_ref/libref_tokenizer.so  the reference's tokenizer.h, compiled as is
                                 from the reference tree (CPU; golden vectors)
  oracle/_ref/libref_model.so    the reference's CUDA forward (qwen_model.cuh,
                                 static_loader.h, config.h) compiled for sm_100a
                                 from the reference tree, linked with cuBLAS

The _ref builds read the reference sources where they lie (REFERENCE_DIR, by
default a directory named "reference" beside the repository) and write only
into oracle/_ref/.  Nothing is copied
into this repository.  When the reference tree is absent (as on a GPU box),
prebuilt _ref libraries that travelled with the snapshot are kept.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("REFERENCE_DIR") or os.path.normpath(os.path.join(HERE, os.pardir, os.pardir, "reference"))
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
OUT = os.path.join(HERE, "liboracle.so")
REF_OUT = os.path.join(HERE, "_ref")


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd):
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force=False):
    src = os.path.join(HERE, "oracle.cpp")
    if force or _stale(OUT, [src, __file__]):
        # -mavx2 -mfma: portable across x86 hosts; no fp contraction so the
        # restatement rounds exactly where its source says.
        _run(["g++", "-O3", "-std=c++17", "-mavx2", "-mfma", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared",
              src, "-o", OUT + ".tmp"])
        os.replace(OUT + ".tmp", OUT)
    if not os.path.isdir(REF):
        return
    os.makedirs(REF_OUT, exist_ok=True)
    samp = os.path.join(REF_OUT, "libref_sampler.so")
    shim = os.path.join(HERE, "ref_sampler_shim.cpp")
    if force or _stale(samp, [shim, os.path.join(REF, "sampler.h"), __file__]):
        _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-I", REF, shim, "-o", samp + ".tmp"])
        os.replace(samp + ".tmp", samp)
    tok = os.path.join(REF_OUT, "libref_tokenizer.so")
    tshim = os.path.join(HERE, "ref_tokenizer_shim.cpp")
    if force or _stale(tok, [tshim, os.path.join(REF, "tokenizer.h"), os.path.join(REF, "config.h"), __file__]):
        _run(["g++", "-O2", "-std=c++17", "-w", "-fPIC", "-shared", "-I", REF, tshim, "-o", tok + ".tmp"])
        os.replace(tok + ".tmp", tok)
    model = os.path.join(REF_OUT, "libref_model.so")
    harness = os.path.join(HERE, "ref_model_harness.cu")
    deps = [harness, __file__] + [os.path.join(REF, f) for f in ("qwen_model.cuh", "static_loader.h", "config.h")]
    if force or _stale(model, deps):
        _run([NVCC, "-O3", "--expt-relaxed-constexpr", "-std=c++17", "-w", "-gencode", "arch=compute_100a,code=sm_100a",
              "-Xcompiler", "-fPIC", "-shared", "-I", REF, harness, "-o", model + ".tmp", "-lcublas"])
        os.replace(model + ".tmp", model)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
