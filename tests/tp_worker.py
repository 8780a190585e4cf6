"""Worker of tests/test_tp_gpu.py: greedy decode of a small model split over every rank of a
torchrun group (tensor / expert parallelism), checked on rank 0 against the CPU oracle.  Prints one JSON
line per rank; exits non-zero on a mismatch."""
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    import datetime

    import torch
    import torch.distributed as dist

    from soso_b200 import decode, synth, tp
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    name = sys.argv[1] if len(sys.argv) > 1 else "TINY"
    steps = int(sys.argv[2]) if len(sys.argv) > 2 else 48
    cfg = getattr(decode, name)
    model = decode.synth_model(cfg, name.lower())  # whole: rank 0's oracle reads every expert
    prompt = synth.rng("prompt", "tp").integers(0, cfg.vocab, 8).astype(np.int32)
    sess = decode.DecodeSession(cfg, model, device=local, group=(rank, world, tp.torch_all_gather()))
    got = sess.greedy(prompt, steps)
    sess.close()
    toks = [None] * world
    dist.all_gather_object(toks, got.tolist())
    ok = all(t == toks[0] for t in toks)
    out = {"rank": rank, "world": world, "ranks_agree": ok}
    if rank == 0:
        from oracle.model import DenseOracle
        want, logits = DenseOracle(cfg, model).greedy(prompt, steps)
        match = bool(np.array_equal(np.array(toks[0], np.int32), want))
        out["matches_oracle"] = match
        if not match:
            d = np.nonzero(np.array(toks[0]) != want)[0]
            out["first_diff"] = int(d[0])
            out["gap_there"] = float(np.sort(logits[d[0]])[-1] - np.sort(logits[d[0]])[-2])
        ok = ok and match
    print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
