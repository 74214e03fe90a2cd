"""Recipe: the reference's own TileLang kernels of the INT8 linear path, built for the
B200 as a second checker (test infrastructure only; nothing in the product loads it).

    python oracle/tilelang_ref.py [--force]

The reference writes the FC2 producer, the row quantiser, the transport codecs and the
row / column epilogues as TileLang kernels (patches/tilelang_swiglu_quant.py:12-64,
tilelang_row_quant.py:27-46, tilelang_transport_tradeoffs.py:26-88,
tilelang_transport_p2.py:15-47, tilelang_column_epilogue.py:11-27,
tilelang_dit_fusion.py:11-37,57-77).  Its factories only accept sm_75 / sm_120 and call
a newer TileLang's compile(); the TileLang installed here (0.1.9) rejects their target
dictionary.  So this recipe runs each factory unmodified from the reference checkout,
takes the kernel definition it hands to tilelang.compile (the call is intercepted in
this process; the reference's sources are not changed or copied), lowers it with the
installed TileLang to CUDA C++ for a generic target (sm_75: plain __syncthreads code),
and compiles that source with nvcc for sm_100a, together with a launcher per kernel,
into

    oracle/_ref/tilelang_ref.cu       generated source (kernels + launchers)
    oracle/_ref/tilelang_ref.json     manifest: per kernel its factory call, parameters
                                      (name, dtype, shape, in factory order), grid,
                                      block and dynamic shared memory
    oracle/_ref/libh3ref_tilelang.so  the build

oracle/_ref/ is git-ignored (generated from the reference) and travels to the GPU box
with the rest of the tree; tests/test_gpu_reference_kernels.py runs the kernels there
next to the B200 path and the C oracle.  TileLang kernels have their shapes baked in,
so the manifest fixes the shapes the tests use.  Needs the reference checkout, TileLang
and nvcc; the GPU box only uses the prebuilt files.
"""
from __future__ import annotations

import hashlib
import json
import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
SRC = OUT / "tilelang_ref.cu"
MANIFEST = OUT / "tilelang_ref.json"
LIB = OUT / "libh3ref_tilelang.so"
# the reference checkout: H3_REFERENCE_DIR, else a `reference` directory beside this repository
REFERENCE = Path(os.environ.get("H3_REFERENCE_DIR", str(HERE.parents[1] / "reference")))

# (name, module under patches/, factory, positional arguments).  Shapes are the ones
# the GPU tests feed; every factory is the reference's own.
KERNELS = [
    ("fc2_stored", "tilelang_swiglu_quant", "fused_kernel", (512, 2048, "float16", "sm_120", "stored")),
    ("fc2_maximum", "tilelang_swiglu_quant", "fused_kernel", (512, 2048, "float16", "sm_120", "maximum")),
    ("fc2_recompute", "tilelang_swiglu_quant", "fused_kernel", (512, 2048, "float16", "sm_120", "recompute")),
    ("quant_rn", "tilelang_row_quant", "quantizer", (512, 2048, 2048, 0, "rn")),
    ("quant_fast", "tilelang_row_quant", "quantizer", (512, 2048, 2048, 0, "fast")),
    ("quant_rn_slice", "tilelang_row_quant", "quantizer", (64, 512, 1024, 256, "rn")),
    ("encode_fp16", "tilelang_transport_tradeoffs", "fp16_codec", (256, 1024, 12, False)),
    ("decode_fp16", "tilelang_transport_tradeoffs", "fp16_codec", (256, 1024, 12, True)),
    ("pack_int8", "tilelang_transport_tradeoffs", "pack_int8", (256, 1024)),
    ("unpack_int8", "tilelang_transport_tradeoffs", "unpack_int8", (256, 1024)),
    ("epilogue_fp16", "tilelang_transport_p2", "epilogue", (256, 1024, "fp16", 12)),
    ("epilogue_int8", "tilelang_transport_p2", "epilogue", (256, 1024, "int8_gather", 0)),
    ("row_gate", "tilelang_dit_fusion", "row_gate_kernel", (256, 1024, 3, 12, "sm_75")),
    ("column_epilogue", "tilelang_column_epilogue", "kernel", (256, 1024, False, "float16", "sm_75")),
    ("modulated_norm", "tilelang_dit_fusion", "norm_kernel", (256, 3072, 3, 1e-6, "sm_75")),
]

_DTYPES = {"float16": "half_t", "float32": "float", "int8": "int8_t", "int32": "int",
           "uint8": "uint8_t"}


def _tilelang_root() -> Path:
    import tilelang
    return Path(tilelang.__file__).resolve().parent


def _capture(module: str, factory: str, args: tuple):
    """Runs the reference factory with tilelang.compile intercepted; returns the
    PrimFunc it built."""
    import tilelang
    captured = {}

    class _Captured(Exception):
        pass

    def intercept(func, *a, **kw):
        captured["func"] = func
        raise _Captured

    real = tilelang.compile
    tilelang.compile = intercept
    try:
        import importlib
        mod = importlib.import_module("patches." + module)
        fn = getattr(mod, factory)
        fn = getattr(fn, "__wrapped__", fn)  # past lru_cache
        try:
            fn(*args)
        except _Captured:
            pass
    finally:
        tilelang.compile = real
    if "func" not in captured:
        raise RuntimeError(f"{module}.{factory}{args} built no kernel")
    return captured["func"]


def _lower(func):
    """CUDA source and launch geometry of one PrimFunc (generic sm_75 lowering)."""
    import tilelang
    from tvm import transform
    from tvm.target import Target
    target = Target("cuda -arch=sm_75")
    with transform.PassContext(config={"tl.enable_async_copy": False}), target:
        art = tilelang.lower(func, target=target)
    kernels = []
    for gv, fn in art.device_mod.functions.items():
        attrs = fn.attrs
        ext = {str(k): int(v) for k, v in attrs["thread_extent"].items()}
        smem = int(attrs["dyn_shared_memory_buf"]) if "dyn_shared_memory_buf" in attrs else 0
        kernels.append({"symbol": str(gv.name_hint), "extent": ext, "smem": smem})
    if len(kernels) != 1:
        raise RuntimeError(f"expected one device kernel, got {len(kernels)}")
    params = []
    for p in func.params:
        buf = func.buffer_map[p]
        params.append({"name": str(buf.name), "dtype": str(buf.dtype),
                       "shape": [int(d) for d in buf.shape]})
    return art.kernel_source, kernels[0], params


def _launcher(name: str, source: str, kern: dict, params: list) -> tuple[str, str]:
    """Renames the kernel to ref_<name>_kernel and writes its launcher
    `int ref_<name>(void** args, void* stream)`, args in the factory's parameter order."""
    sym = kern["symbol"]
    kname = f"ref_{name}_kernel"
    source = re.sub(r"\b%s\b" % re.escape(sym), kname, source)
    m = re.search(r'extern "C" __global__ void[^(]*\b%s\(([^)]*)\)' % kname, source)
    if m is None:
        raise RuntimeError(f"kernel signature of {name} not found")
    sig = [a.strip() for a in m.group(1).split(",") if a.strip()]
    order = {p["name"]: i for i, p in enumerate(params)}
    casts = []
    for a in sig:
        pname = a.split()[-1].lstrip("*")
        ctype = a[: a.rfind(pname)].replace("__restrict__", "").strip()
        casts.append(f"({ctype})args[{order[pname]}]")
    e = kern["extent"]
    grid = (e.get("blockIdx.x", 1), e.get("blockIdx.y", 1), e.get("blockIdx.z", 1))
    block = (e.get("threadIdx.x", 1), e.get("threadIdx.y", 1), e.get("threadIdx.z", 1))
    smem = kern["smem"]
    launch = f'''
extern "C" int ref_{name}(void** args, void* stream) {{
  if ({smem} > 48 * 1024 &&
      cudaFuncSetAttribute({kname}, cudaFuncAttributeMaxDynamicSharedMemorySize, {smem}) != cudaSuccess)
    return 1;
  {kname}<<<dim3({grid[0]}, {grid[1]}, {grid[2]}), dim3({block[0]}, {block[1]}, {block[2]}), {smem},
           (cudaStream_t)stream>>>({", ".join(casts)});
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}}
'''
    return source, launch, {"grid": list(grid), "block": list(block), "smem": smem}


def _digest() -> str:
    h = hashlib.sha256(Path(__file__).read_bytes())
    for _, module, _, _ in KERNELS:
        p = REFERENCE / "patches" / f"{module}.py"
        h.update(p.read_bytes() if p.exists() else b"")
    return h.hexdigest()


def available() -> bool:
    if not (REFERENCE / "patches").is_dir():
        return False
    try:
        import tilelang  # noqa: F401
    except Exception:
        return False
    return shutil.which("nvcc") is not None or Path("/usr/local/cuda/bin/nvcc").exists()


def build(force: bool = False) -> Path | None:
    """Generates and compiles the reference kernels; returns the library path, or None
    when the reference checkout, TileLang or nvcc is missing (the GPU box: it uses the
    files built here)."""
    stamp = OUT / "tilelang_ref.stamp"
    if not available():
        return LIB if LIB.exists() else None
    digest = _digest()
    if not force and LIB.exists() and MANIFEST.exists() and stamp.exists() \
            and stamp.read_text() == digest:
        return LIB
    OUT.mkdir(parents=True, exist_ok=True)
    if str(REFERENCE) not in sys.path:
        sys.path.insert(0, str(REFERENCE))
    bodies, launchers, manifest = [], [], {}
    for name, module, factory, args in KERNELS:
        func = _capture(module, factory, args)
        source, kern, params = _lower(func)
        source, launch, geom = _launcher(name, source, kern, params)
        bodies.append(f"// ---- {module}.{factory}{args}\n" + source)
        launchers.append(launch)
        manifest[name] = {"factory": f"patches/{module}.py:{factory}", "args": list(args),
                          "params": params, **geom}
    unit = ("// Generated by oracle/tilelang_ref.py from the reference's TileLang kernels.\n"
            "// Test infrastructure only.\n" + "\n".join(bodies) + "\n".join(launchers))
    SRC.write_text(unit)
    MANIFEST.write_text(json.dumps(manifest, indent=1))
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    tl = _tilelang_root()
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O3",
           "-Xcompiler", "-fPIC", "-shared", "-w", "-I" + str(tl / "src"),
           "-I" + str(tl / "3rdparty" / "cutlass" / "include"), str(SRC), "-o",
           str(LIB.with_suffix(".so.tmp"))]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("reference kernel build failed:\n" + r.stdout[-4000:] + r.stderr[-4000:])
    os.replace(LIB.with_suffix(".so.tmp"), LIB)
    stamp.write_text(digest)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
