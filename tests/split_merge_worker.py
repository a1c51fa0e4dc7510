"""Child process of test_gpu_split_merge.py: runs one fixed workload through the
C-ABI and saves every output.  MS_SPLITK_GLOBAL in the environment picks how
split-K partials and attention splits are merged (thread-block clusters by
default, global memory and arrival tickets with MS_SPLITK_GLOBAL=1)."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main(out_path):
    import torch

    from mojostream_b200.model import small_spec, synth_weights
    from mojostream_b200.runtime import Context, KVCache, Model, Q4Weight

    ctx = Context(0)
    out = {}
    # decode projections: k-segments 2..8 (cluster-sized) and 16 (global either way)
    rng = np.random.default_rng(11)
    for (M, K, N) in [(4, 2560, 2560), (4, 2048, 2560), (8, 10240, 2560), (4, 1024, 128)]:
        W = rng.integers(0, 256, size=(K, N // 2), dtype=np.uint8)
        A = rng.standard_normal((M, K)).astype(np.float32)
        w = Q4Weight(ctx, W, K, N, 0.01)
        C = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        w.gemm(torch.from_numpy(A).cuda(), C)
        torch.cuda.synchronize()
        out[f"gemm_{M}_{K}_{N}"] = C.cpu().numpy()
        w.close()
    # a hybrid model: 4 sequences, so a decode attention row has 8 (sliding) to
    # 16 (full) splits in one cluster
    spec = small_spec(vocab=4096, n_layers=6, window=64)
    w = synth_weights(spec, seed=7, symmetric=True)
    model = Model(ctx, spec, w, max_rows=64)
    kv = KVCache(ctx, model, 4, 256, slide_cap=64 + 64)
    prompts = [list(rng.integers(0, 4096, size=L)) for L in (40, 23, 57, 9)]
    ids = sum(prompts, [])
    seq = sum([[s] * len(p) for s, p in enumerate(prompts)], [])
    pos = sum([list(range(len(p))) for p in prompts], [])
    first = model.prefill(kv, ids, seq, pos)
    gen = model.generate(kv, first, [0, 1, 2, 3], [len(p) for p in prompts], 6)
    out["first"] = np.array(first)
    out["gen"] = np.array(gen)
    x = rng.standard_normal((4, spec.hidden)).astype(np.float32)
    for layer in (4, 5):  # a sliding and a full layer
        xg = torch.from_numpy(x).cuda()
        model.layer_forward(layer, xg, kv, [0, 1, 2, 3], [len(p) + 6 for p in prompts])
        torch.cuda.synchronize()
        out[f"layer{layer}"] = xg.cpu().numpy()
    np.savez(out_path, **out)


if __name__ == "__main__":
    main(sys.argv[1])
