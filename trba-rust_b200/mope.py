"""MoPE length-bucket inference serving on B200s.

The reference trains one TRBA expert per label-length bucket
(scripts/run_len_buckets.sh, README.md:51-60) and serves them with a learned
router and an aggregator (src/moe.rs, later snapshot).  This module serves
the bucketed experts the way the benchmark defines the workload: every line
is routed to the expert of its length bucket on the host, experts are placed
on the GPUs of one box by greedy bin-packing of their expected work, and each
GPU decodes its lines greedily with libtrba_b200's inference path
(trba_model_infer).  No tensor crosses GPUs; only the decoded token lists
are gathered.

    experts = default_experts()
    plan = place(experts, lines_per_bucket, world)      # expert -> rank
"""
from __future__ import annotations

import dataclasses
from typing import Sequence


@dataclasses.dataclass(frozen=True)
class Expert:
    name: str
    lo: int          # shortest label length routed here
    hi: int          # longest label length routed here
    img_w: int       # expert input width (images are 32 x img_w)
    max_len: int     # decoder steps = max_len + 1


# README.md:51-60 of the reference: 9 buckets, widths and max_len per bucket.
DEFAULT_BUCKETS = [
    ("bucket_04_04", 4, 4, 64, 4), ("bucket_05_05", 5, 5, 96, 5), ("bucket_06_06", 6, 6, 96, 6),
    ("bucket_07_07", 7, 7, 128, 7), ("bucket_08_08", 8, 8, 128, 8), ("bucket_09_09", 9, 9, 160, 9),
    ("bucket_10_10", 10, 10, 160, 10), ("bucket_11_12", 11, 12, 192, 12), ("bucket_13_40", 13, 40, 256, 40),
]


def default_experts() -> list[Expert]:
    return [Expert(*b) for b in DEFAULT_BUCKETS]


def route(lengths: Sequence[int], experts: Sequence[Expert]) -> list[int]:
    """Expert index of every line: the bucket containing its label length;
    shorter lines than the first bucket go to the first, longer than the last
    to the last."""
    out = []
    for n in lengths:
        k = len(experts) - 1
        for i, e in enumerate(experts):
            if n <= e.hi:
                k = i
                break
        out.append(k)
    return out


def expected_work(e: Expert, lines: int) -> float:
    """Relative cost of decoding `lines` lines with expert e: the CNN scales
    with the image width, the decoder with its steps."""
    return float(lines) * (e.img_w + 8.0 * (e.max_len + 1))


def place(experts: Sequence[Expert], lines_per_expert: Sequence[int], world: int) -> list[int]:
    """Rank of every expert: largest expected work first, each onto the rank
    with the least work so far (greedy bin-packing); ties go to the lower
    rank."""
    if world < 1:
        raise ValueError("world must be >= 1")
    load = [0.0] * world
    rank = [0] * len(experts)
    order = sorted(range(len(experts)), key=lambda i: (-expected_work(experts[i], lines_per_expert[i]), i))
    for i in order:
        r = min(range(world), key=lambda j: (load[j], j))
        rank[i] = r
        load[r] += expected_work(experts[i], lines_per_expert[i])
    return rank


def synthetic_lengths(n: int, seed: int, max_len: int = 32) -> list[int]:
    """Label lengths with the corpus quantiles the reference documents
    (README.md:48-49: median 5, p90 11, max 32): log-normal, rounded and
    clipped to [1, max_len]."""
    import numpy as np
    rng = np.random.default_rng(seed)
    mu = np.log(5.0)
    sigma = (np.log(11.0) - mu) / 1.2815515655446004  # p90 of the standard normal
    v = np.rint(np.exp(rng.normal(mu, sigma, n)))
    return np.clip(v, 1, max_len).astype(int).tolist()


class ExpertRunner:
    """One expert on the current GPU: an inference-only int8 model (weights
    quantised per output channel, no gradient or optimiser buffers) sized
    for `batch` lines per decoding call; greedy decoding of device image
    batches.  per_channel=False gives the reference's per-tensor scales."""

    def __init__(self, expert: Expert, batch: int, seed: int, per_channel: bool = True):
        from .data import init_params
        from .model import Config, QatModel
        self.expert, self.batch = expert, batch
        self.cfg = Config(img_w=expert.img_w, max_len=expert.max_len, batch=batch,
                          wq_per_channel=int(per_channel), inference_only=1)
        self.model = QatModel(self.cfg)
        self.model.set_params(init_params(self.model.manifest(), self.cfg, seed))

    def decode_steps(self, imgs, stream=None) -> list:
        """Per-step argmax tokens ([steps, n] each) of device images
        [n, 3, 32, img_w], one array per decoding batch of the runner."""
        return [self.model.infer(imgs[s:s + self.batch], stream=stream) for s in range(0, imgs.shape[0], self.batch)]

    def decode(self, imgs, stream=None) -> list[list[int]]:
        """Token lists of device images, the reference's output rule applied
        per decoding batch."""
        out = []
        for st in self.decode_steps(imgs, stream):
            out.extend(decode_rule(st, self.cfg.eos))
        return out

    def close(self):
        self.model.close()


def decode_rule(step_tokens, eos: int) -> list[list[int]]:
    """The reference's greedy output (src/attn.rs:423-443) from per-step
    argmax tokens [steps, n] of ONE decoding batch: eos is not emitted and
    decoding stops after the first step at which every line produced eos."""
    steps, n = step_tokens.shape
    last = steps - 1
    for s in range(steps):
        if all(int(step_tokens[s, b]) == eos for b in range(n)):
            last = s
            break
    return [[int(step_tokens[s, b]) for s in range(last + 1) if int(step_tokens[s, b]) != eos] for b in range(n)]
