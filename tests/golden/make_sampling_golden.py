"""Golden vectors for the fused sampling kernel, from the reference's own code.

Runs the reference's ``_sample_topk_kernel`` (qwen3/sampling.py:112-178) and
Triton's ``tl.rand`` under Triton's CPU interpreter (TRITON_INTERPRET=1; the
reference pins Triton 2.2.0 in PERFORMANCE.md:10, this container has 3.6.0),
on seeded logits with per-row temperature / top-k / top-p, after the
reference's batched ``torch.topk`` (qwen3/sampling.py:215-216).

    python tests/golden/make_sampling_golden.py --reference <reference checkout>
"""

import argparse
import json
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"   # must precede every triton.jit decoration

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import synth  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("QWEN3_REFERENCE"))
    args = ap.parse_args()
    if not args.reference or not os.path.isdir(args.reference):
        sys.exit("make_sampling_golden.py: pass --reference <path>")
    sys.path.insert(0, args.reference)
    import torch
    import triton
    import triton.language as tl
    from qwen3 import sampling as S
    torch.set_num_threads(1)

    # ---- Philox stream of tl.rand(seed, offsets)
    @triton.jit
    def rand_kernel(out_ptr, seed, n, BLOCK: tl.constexpr):
        offs = tl.arange(0, BLOCK)
        u = tl.rand(seed, offs)
        bits = tl.randint(seed, offs)
        tl.store(out_ptr + offs, u, mask=offs < n)
        tl.store(out_ptr + BLOCK + offs, bits.to(tl.float32, bitcast=True), mask=offs < n)

    seeds = [1234, 0x7FFFFFFF, 99991]
    rand_u, rand_bits = [], []
    for sd in seeds:
        buf = torch.zeros(2 * 4096, dtype=torch.float32)
        rand_kernel[(1,)](buf, sd, 4096, BLOCK=4096)
        rand_u.append(buf[:4096].numpy().copy())
        rand_bits.append(buf[4096:].numpy().view(np.uint32).copy())

    # ---- the sampling kernel on seeded logits, one row per parameter combination
    temps = [0.0, 0.5, 1.0, 1.3]
    ks = [1, 5, 50, 200, 1000]
    ps = [1.0, 0.9, 0.5]
    combos = [(t, k, p) for t in temps for k in ks for p in ps]     # 60 rows
    B, V = len(combos), 4096
    logits = synth.det_normal(901, (B, V)) * np.float32(3.0)
    lt = torch.from_numpy(logits)
    temp = [c[0] for c in combos]
    kk = [c[1] for c in combos]
    pp = [c[2] for c in combos]
    seed = 1234
    max_k = min(max(kk), V)
    params = torch.tensor([temp, [min(k, V) for k in kk], pp,
                           [1.0 if t <= 0 else 0.0 for t in temp]], dtype=torch.float32)
    vals, idx = torch.topk(lt, max_k, dim=-1, largest=True, sorted=True)
    out = torch.empty(B, dtype=torch.int64)
    block_k = max(16, triton.next_power_of_2(max_k))
    S._sample_topk_kernel[(B,)](vals, idx, params, out, vals.stride(0), idx.stride(0), B, max_k,
                                seed, BLOCK_K=block_k, num_warps=1)
    meta = dict(case="sampling", seed_logits=901, scale=3.0, B=B, V=V, seed=seed, max_k=max_k,
                block_k=block_k, temperature=temp, top_k=kk, top_p=pp, rand_seeds=seeds,
                triton=triton.__version__,
                reference_fn="qwen3/sampling.py:_sample_topk_kernel after torch.topk, "
                             "Triton interpreter")
    np.savez_compressed(os.path.join(HERE, "sampling.npz"), meta=np.array(json.dumps(meta)),
                        tokens=out.numpy(), rand_u=np.stack(rand_u), rand_bits=np.stack(rand_bits))
    print("sampling: ok", out[:8].tolist())


if __name__ == "__main__":
    main()
