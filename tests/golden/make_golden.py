"""Generates the golden fixtures in tests/golden/ by running the reference crate's own CUDA
kernels (oracle/_ref/libref_moe.so, built by oracle/build_ref.sh) on seeded inputs.  Needs a
GPU; run from the repository root:  python tests/golden/make_golden.py OUTPUT_DIR
The fixtures pin the CPU oracle (tests/test_oracle.py) to the reference's actual outputs."""
import os
import sys
import zlib

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [ROOT, os.path.join(ROOT, "tests")]

import oracle  # noqa: E402
from oracle import refkernels  # noqa: E402
from moe_testlib import from_torch, moe_case, to_torch  # noqa: E402

DT = {"f16": 0, "bf16": 1, "f32": 2}


def main(out_dir):
    os.makedirs(out_dir, exist_ok=True)
    # router (kernels/topk_softmax.cu)
    for T, E, k in [(8, 4, 2), (64, 8, 2), (96, 128, 8), (40, 256, 4), (33, 16, 3)]:
        logits = oracle.randn(1000 + T + E, (T, E))
        w, i, s = refkernels.topk_softmax(torch.from_numpy(logits).cuda(), k)
        np.savez_compressed(os.path.join(out_dir, f"router_T{T}_E{E}_k{k}.npz"), logits=logits,
                            k=k, weights=w.cpu().numpy(), indices=i.cpu().numpy(),
                            token_expert_indices=s.cpu().numpy())
    # preprocessing (kernels/preprocessing.cuh, single-CTA path)
    for T, k, E in [(512, 2, 8), (700, 8, 128), (300, 3, 5)]:
        rng = np.random.default_rng(T + k + E)
        idx = rng.integers(0, E, size=(T, k)).astype(np.uint32)
        w = rng.standard_normal((T, k)).astype(np.float32)
        off, st, sw = refkernels.preprocessing(torch.from_numpy(idx.view(np.int32)).cuda(),
                                               torch.from_numpy(w).cuda(), E)
        np.savez_compressed(os.path.join(out_dir, f"prep_T{T}_k{k}_E{E}.npz"), indices=idx,
                            weights=w, E=E, offsets=off.cpu().numpy(),
                            sorted_token_ids=st.cpu().numpy(), sorted_weights=sw.cpu().numpy())
    # fused MoE on the reference paths that launch (f32 FFMA, direct f16/bf16, small wmma)
    cases = [
        # name, dtype, moe_type, act, T, H, I, E, k, round_dtype, rtol
        ("f32_nomic_silu", "f32", 1, 0, 16, 16, 64, 8, 2, "f32", 1e-4),
        ("f32_qwen3_silu", "f32", 0, 0, 32, 64, 256, 8, 2, "f32", 1e-4),
        ("f32_nomic_gelu", "f32", 1, 1, 64, 32, 128, 8, 2, "f32", 1e-4),
        ("f32_qwen3_relu", "f32", 0, 2, 48, 32, 96, 4, 3, "f32", 1e-4),
        ("bf16_qwen3_direct", "bf16", 0, 0, 4, 64, 256, 8, 2, "bf16", 1e-2),
        ("f16_nomic_direct", "f16", 1, 0, 32, 64, 256, 8, 1, "f16", 1e-2),
        ("f16_qwen3_direct_gelu", "f16", 0, 1, 20, 128, 256, 8, 2, "f16", 1e-2),
        ("f16_qwen3_small_gemm", "f16", 0, 0, 48, 64, 256, 8, 1, "f16", 1e-2),
        ("bf16_nomic_small_gemm", "bf16", 1, 0, 60, 64, 256, 8, 1, "bf16", 1e-2),
    ]
    for name, dtype, mt, act, T, H, I, E, k, rd, rtol in cases:
        c = moe_case(zlib.crc32(name.encode()) % 1000, T=T, H=H, I=I, E=E, k=k, moe_type=mt, dtype=dtype,
                     wstd=0.1)
        out, err = refkernels.fused_moe(
            to_torch(c["x"], dtype), to_torch(c["gate"], dtype), to_torch(c["up"], dtype),
            None if c["down"] is None else to_torch(c["down"], dtype),
            torch.from_numpy(c["w"]).cuda(), torch.from_numpy(c["idx"]).cuda(), E, k, act, mt,
            DT[dtype])
        if err != 0:
            print(f"{name}: reference launch failed with cuda error {err}; fixture skipped")
            continue
        d = dict(x=c["x"], gate=c["gate"], up=c["up"], w=c["w"], idx=c["idx"],
                 out=from_torch(out, dtype), dtype=dtype, moe_type=mt, act=act, round_dtype=rd,
                 rtol=rtol)
        if c["down"] is not None:
            d["down"] = c["down"]
        np.savez_compressed(os.path.join(out_dir, f"moe_{name}.npz"), **d)
    print("fixtures written to", out_dir)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
