"""TEST INFRASTRUCTURE ONLY. Compile the reference's own CUDA kernels into oracle/_ref/ref_kernels.cubin.

    python oracle/build_ref.py [/path/to/ComfyUI-Drama3]

Without an argument the checkout is taken from the DRAMA3_REFERENCE environment variable, else from the
"reference_path" entry of BASELINE.json at the repository root; with none of these nothing is built.

The reference keeps its kernels as one CUDA C string (drama3/kernels.py:14-588, `SOURCE`) and compiles it at run
time with NVRTC for the current device (drama3/kernels.py:593-596, through torch.cuda._compile_kernel, which adds
-D__CUDA_NO_HALF_OPERATORS__ and friends and nothing that changes float code). This recipe reads that string from
the reference checkout, writes it to a temporary directory outside this repository, and compiles it with nvcc for
sm_100 with the same defines; only the cubin lands in oracle/_ref/ (git-ignored; it travels to the GPU box with
the working tree). Nothing of the reference's source is kept.
"""
import ast
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
CUBIN = OUT_DIR / "ref_kernels.cubin"
DEFINES = ["-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__", "-D__CUDA_NO_BFLOAT16_CONVERSIONS__",
           "-D__CUDA_NO_HALF2_OPERATORS__"]


def reference_source(root):
    """The SOURCE string of drama3/kernels.py, read by parsing the file (no import of the reference)."""
    tree = ast.parse((Path(root) / "drama3" / "kernels.py").read_text())
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(getattr(t, "id", None) == "SOURCE" for t in node.targets):
            return ast.literal_eval(node.value)
    raise RuntimeError("SOURCE not found in drama3/kernels.py")


def reference_root():
    """The reference checkout named by DRAMA3_REFERENCE or by BASELINE.json's "reference_path", or None."""
    if os.environ.get("DRAMA3_REFERENCE"):
        return Path(os.environ["DRAMA3_REFERENCE"])
    baseline = HERE.parent / "BASELINE.json"
    if baseline.exists():
        path = json.loads(baseline.read_text()).get("reference_path")
        if path:
            return Path(path)
    return None


def build(root=None, force=False):
    """Build the cubin when the reference checkout is present; returns its path (or None without the checkout)."""
    root = root or reference_root()
    if root is None:
        return CUBIN if CUBIN.exists() else None
    kernels = Path(root) / "drama3" / "kernels.py"
    if not kernels.exists():
        return CUBIN if CUBIN.exists() else None
    if CUBIN.exists() and not force and CUBIN.stat().st_mtime >= kernels.stat().st_mtime:
        return CUBIN
    OUT_DIR.mkdir(exist_ok=True)
    with tempfile.TemporaryDirectory() as tmp:
        src = Path(tmp) / "reference_kernels.cu"
        src.write_text(reference_source(root))
        out = Path(tmp) / "ref_kernels.cubin"
        nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
        subprocess.run([nvcc, "-cubin", "-arch=sm_100", "-O3", *DEFINES, "-o", str(out), str(src)], check=True,
                       stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        os.replace(out, CUBIN)
    return CUBIN


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, force=True))
