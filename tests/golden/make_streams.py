"""Make the token-stream fixture the benchmark replays (both arms read the same streams).

    python tests/golden/make_streams.py --config 3 --out tests/golden/streams_paths100k.npz

Needs a CUDA GPU: the streams are constrained decodes sampled with the engine's own masks
(xgraph_b200.synthetic.sample_streams, a seeded span-biased walk), `--streams` rows of
`--steps` tokens each, plus one seeded replay length per stream, uniform in the
configuration's length range.  The fixture is checked on the CPU against the oracle
(tests/test_streams_fixture.py: every token of every stream must be allowed), so the
reference arm of bench.py can replay it without loading the engine library.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--config", type=int, default=3)
    parser.add_argument("--seed", type=int, default=None, help="world seed (default: the config number)")
    parser.add_argument("--streams", type=int, default=512)
    parser.add_argument("--steps", type=int, default=None, help="tokens per stream (default: the longest length)")
    parser.add_argument("--out", type=Path, required=True)
    args = parser.parse_args()

    import torch

    from xgraph_b200.engine import Engine
    from xgraph_b200.synthetic import build_workload, sample_streams

    workload = build_workload(args.config, args.seed)
    cfg = workload.config
    seed = args.config if args.seed is None else args.seed
    steps = args.steps or cfg.lengths[1]
    engine = Engine(workload.index, workload.served, workload.syntax, args.streams, **cfg.options)
    tokens, counts, _ = sample_streams(engine, workload.served, workload.syntax, workload.world, args.streams,
                                       steps, seed=seed + 1000)
    torch.cuda.synchronize()
    lengths = np.random.default_rng(seed + 2000).integers(cfg.lengths[0], cfg.lengths[1] + 1, size=args.streams)
    np.savez_compressed(
        args.out, tokens=tokens.cpu().numpy().astype(np.uint32), lengths=lengths.astype(np.int32),
        allowed=counts.cpu().numpy().astype(np.int32), config=np.int32(args.config), seed=np.int32(seed),
        vocab=np.int32(workload.served.vocab_size), fingerprint=np.array(workload.served.fingerprint))
    print(f"{args.out}: {args.streams} streams x {steps} tokens, config {args.config}")


if __name__ == "__main__":
    main()
