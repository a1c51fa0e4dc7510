"""One rank of the tensor-parallel GPU test (tests/test_tp.py launches it).

Env: RANK, WORLD_SIZE, MASTER_PORT.  argv[1]: output path prefix.  Builds the
small hybrid model sharded over WORLD_SIZE GPUs, prefills two prompts,
decodes four greedy steps and runs one teacher-forced layer, then a sampled
generation; writes the ids and the layer output as JSON (rank 0 and 1 must
agree with the oracle).
"""
import datetime
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main(prefix):
    import numpy as np
    import torch
    import torch.distributed as dist

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{os.environ['MASTER_PORT']}",
                            rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    from mojostream_b200.model import small_spec, synth_weights
    from mojostream_b200.runtime import Context, KVCache, Model
    from mojostream_b200.tp import tp_setup

    spec = small_spec(vocab=4096, n_layers=6, window=32)
    w = synth_weights(spec, seed=1234, symmetric=True)
    ctx = Context(rank)
    tp_setup(ctx)
    model = Model(ctx, spec, w, max_rows=16)
    kv = KVCache(ctx, model, 2, 64, slide_cap=48)
    prompts = [[11, 402, 7, 3999, 58], [1, 2, 3]]
    ids = sum(prompts, [])
    seq = [0] * 5 + [1] * 3
    pos = list(range(5)) + list(range(3))
    first = model.prefill(kv, ids, seq, pos)
    gen = model.generate(kv, first, [0, 1], [5, 3], 4)

    kv2 = KVCache(ctx, model, 2, 64, slide_cap=48)
    x = np.random.default_rng(0).standard_normal((2, spec.hidden)).astype(np.float32)
    xg = torch.from_numpy(x).cuda()
    model.layer_forward(5, xg, kv2, [0, 1], [0, 0])
    torch.cuda.synchronize()
    # rows > 8: the tensor-core projections with the all-reduce inside their
    # epilogue (a 16-row prefill chunk, then 5 rows; a 12-row layer)
    kv3 = KVCache(ctx, model, 2, 64, slide_cap=48)
    long_prompts = [[(37 * i + 11) % 4096 for i in range(12)], [(91 * i + 5) % 4096 for i in range(9)]]
    ids3 = sum(long_prompts, [])
    seq3 = [0] * 12 + [1] * 9
    pos3 = list(range(12)) + list(range(9))
    first3 = model.prefill(kv3, ids3, seq3, pos3)
    gen3 = model.generate(kv3, first3, [0, 1], [12, 9], 3)
    kv4 = KVCache(ctx, model, 2, 64, slide_cap=48)
    x12 = np.random.default_rng(1).standard_normal((12, spec.hidden)).astype(np.float32)
    xg12 = torch.from_numpy(x12).cuda()
    model.layer_forward(3, xg12, kv4, [0] * 12, list(range(12)))
    torch.cuda.synchronize()
    # sampled token loop (temperature + repetition penalty, then greedy +
    # penalty): the vocabulary shards combine through the sampler's collectives
    sampled = {}
    for key, (T, pen) in {"samp": (0.7, 1.2), "samp_greedy": (0.0, 1.3)}.items():
        model.set_sampling(T, pen, 2024)
        kv5 = KVCache(ctx, model, 2, 64, slide_cap=48)
        f5 = model.prefill(kv5, ids, seq, pos)
        g5 = model.generate(kv5, f5, [0, 1], [5, 3], 6)
        sampled[key] = [[int(v) for v in f5]] + np.asarray(g5).tolist()
        kv5.close()
    model.set_sampling()
    out = {"first": [int(v) for v in first], "gen": np.asarray(gen).tolist(), **sampled,
           "layer5": xg.cpu().numpy().astype(np.float64).tolist(),
           "first3": [int(v) for v in first3], "gen3": np.asarray(gen3).tolist(),
           "layer3_12": xg12.cpu().numpy().astype(np.float64).tolist()}
    kv4.close()
    kv3.close()
    with open(f"{prefix}.{rank}.json", "w") as f:
        json.dump(out, f)
    kv2.close()
    kv.close()
    model.close()
    ctx.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
