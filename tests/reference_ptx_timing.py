"""Times the reference's own PTX (rescaled public packages) against this backend on the B200.

    python tests/reference_ptx_timing.py [--repeat R]

Test infrastructure: prints one JSON object per package with the CUDA-event
mean of R launches (after one warm-up) for the reference PTX under its
meta.json geometry and for this backend's kernel on the same device
buffers, and the algorithmic GB/s of each.  The FP32 GEMM and attention
packages are timed at their own (small) shapes, kernel launches only (the
launcher's zeroing of split-K outputs is excluded for both).
"""
import argparse
import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))
sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from lazy_compiler_b200.compiler import compile_file  # noqa: E402
from lazy_compiler_b200.runtime import launch  # noqa: E402
from refptx import REF, RefKernel, manifest_rescaled  # noqa: E402
from test_gpu_reference_ptx_config import device_inputs  # noqa: E402

BYTES = {"r02_big_sum": 4 << 24, "r03_mean": 4 << 24, "p01_vector_add": 12 << 28,
         "p02_scale_shift": 8 << 28, "p03_relu_mul": 12 << 28, "phase9_gelu_erf_tail": 8 << 28,
         "r04_row_sum": 4 * 16384 * 4096 + 4 * 16384, "f01_rmsnorm": 8 * 16384 * 4096 + 4 * 4096,
         "f02_row_softmax": 8 * 16384 * 4096, "f03_l2norm": 8 * 16384 * 4096}


def time_ms(fn, repeat):
    import torch
    fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(repeat):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / repeat


def main():
    import torch
    ap = argparse.ArgumentParser()
    ap.add_argument("--repeat", type=int, default=5)
    args = ap.parse_args()
    stream = torch.cuda.current_stream().cuda_stream
    for name, row in sorted(manifest_rescaled().items()):
        kernel = RefKernel(name, rescaled=True)
        _, buffers = kernel.run(device_inputs(kernel, seed=1), keep=True)
        ptrs = {n: t.data_ptr() for n, t in buffers.items()}
        (ir,) = sorted((REF.parent.parent / row["package"]).glob("*.ir.json"))
        plan = compile_file(ir)
        ref_ms = time_ms(lambda: kernel.launch(ptrs, stream), args.repeat)
        our_ms = time_ms(lambda: launch(plan, ptrs, stream), args.repeat)
        gb = BYTES[name] / 1e9
        print(json.dumps({"package": name, "rescaled": True, "reference_ptx_ms": round(ref_ms, 4),
                          "ours_ms": round(our_ms, 4), "reference_ptx_gbs": round(gb / ref_ms * 1e3, 1),
                          "ours_gbs": round(gb / our_ms * 1e3, 1), "speedup": round(ref_ms / our_ms, 2),
                          "grid": kernel.kernel_meta["grid"], "block": kernel.kernel_meta["block"]}), flush=True)
    native(args.repeat)


NATIVE = {"m01_matmul_512": 2 * 512 ** 3, "m02_matmul_rect": 2 * 128 * 64 * 256,
          "phase9_bias_gelu_gemm": 2 * 33 * 47 * 65, "a01_attention": 4 * 64 * 64 * 64,
          "a02_attention_128": 4 * 128 * 128 * 32, "phase9_gelu_attention": 2 * 11 * 37 * (17 + 13)}


def native(repeat):
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    from refptx import manifest
    rows = manifest()
    for name, flops in NATIVE.items():
        if name not in rows or "error" in rows[name]:
            continue
        kernel = RefKernel(name)
        _, buffers = kernel.run(device_inputs(kernel, seed=1), keep=True)
        ptrs = {n: t.data_ptr() for n, t in buffers.items()}
        (ir,) = sorted((REF.parent.parent / "tests" / "golden" / "packages" / name).glob("*.ir.json"))
        plan = compile_file(ir)
        ref_ms = time_ms(lambda: kernel.launch(ptrs, stream), repeat)
        our_ms = time_ms(lambda: launch(plan, ptrs, stream), repeat)
        print(json.dumps({"package": name, "rescaled": False, "reference_ptx_us": round(ref_ms * 1e3, 2),
                          "ours_us": round(our_ms * 1e3, 2), "ours_path": plan["op"],
                          "reference_ptx_gflops": round(flops / ref_ms / 1e6, 1),
                          "ours_gflops": round(flops / our_ms / 1e6, 1), "speedup": round(ref_ms / our_ms, 2),
                          "grid": kernel.kernel_meta["grid"], "block": kernel.kernel_meta["block"]}), flush=True)


if __name__ == "__main__":
    main()
