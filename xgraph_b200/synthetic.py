"""Seeded synthetic workloads: KGs, served tokenizers and constrained token streams.

No public dataset is involved.  The generator is the one the measurement plan fixes:
entity labels are 1-3 capitalised words of 2-4 syllables from a fixed syllable list
(homonyms included on purpose), relation labels are distinct lowercase words, triples
are uniform (or, for the path-mode config, with Zipf out-degrees), and the served
tokenizer is a byte-level BPE trained by the `tokenizers` library on the label corpus
plus seeded prose, padded with non-special added tokens to the exact vocabulary size.

Token streams are constrained decodes: `sample_streams` runs the engine itself as the
sampler's constraint, one step at a time on the GPU, choosing for every row a token its
mask allows, biased toward whole spans (open, take separators and closers, escape now
and then) the way the reference's agreement harness walks the oracle
(tests/test_engine.py:1903-1960).  Every token is therefore allowed by construction.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

CONSONANTS = "bcdfghjklmnprstvz"
VOWELS = "aeiou"
SYLLABLES = [c + v for c in CONSONANTS for v in VOWELS] + ["an", "el", "or", "ul", "is", "en", "ay", "oo"]


def _words(rng: np.random.Generator, n: int, syllables=(2, 4), capital=True) -> np.ndarray:
    counts = rng.integers(syllables[0], syllables[1] + 1, size=n)
    picks = rng.integers(0, len(SYLLABLES), size=int(counts.sum()))
    table = np.array(SYLLABLES, dtype=object)
    parts = table[picks]
    out = np.empty(n, dtype=object)
    at = 0
    for i, c in enumerate(counts.tolist()):
        w = "".join(parts[at: at + c])
        out[i] = w.capitalize() if capital else w
        at += c
    return out


def _labels(rng: np.random.Generator, n: int, words=(1, 3)) -> list[str]:
    counts = rng.integers(words[0], words[1] + 1, size=n)
    pool = _words(rng, int(counts.sum()))
    out, at = [], 0
    for c in counts.tolist():
        out.append(" ".join(pool[at: at + c]))
        at += c
    return out


@dataclass
class World:
    entities: list[tuple[str, list[str]]]
    relations: list[tuple[str, list[str]]]
    triples: np.ndarray  # int64 (n, 3) positions
    sitelinks: np.ndarray
    prose: list[str] = field(default_factory=list)


def synthetic_world(seed: int, entities: int, relations: int, triples: int, *, labels=(1, 1),
                    homonyms: float = 0.03, zipf: float | None = None) -> World:
    rng = np.random.default_rng(seed)
    label_counts = rng.integers(labels[0], labels[1] + 1, size=entities)
    pool = _labels(rng, int(label_counts.sum()))
    # homonyms: reuse an earlier label for a share of the labels
    reuse = rng.random(len(pool)) < homonyms
    sources = rng.integers(0, np.maximum(np.arange(len(pool)), 1))
    for i in np.flatnonzero(reuse).tolist():
        if i > 0:
            pool[i] = pool[int(sources[i])]
    ents, at = [], 0
    for n, c in enumerate(label_counts.tolist()):
        ents.append((f"Q{n}", list(dict.fromkeys(pool[at: at + c]))))
        at += c
    names: list[str] = []
    seen: set[str] = set()
    while len(names) < relations:
        for w in _words(rng, relations, syllables=(2, 3), capital=False).tolist():
            if w not in seen and len(names) < relations:
                seen.add(w)
                names.append(w)
    rels = [(f"P{n}", [w]) for n, w in enumerate(names)]
    if zipf is None:
        subjects = rng.integers(0, entities, size=triples)
    else:
        weights = 1.0 / np.arange(1, entities + 1) ** zipf
        order = rng.permutation(entities)
        subjects = order[rng.choice(entities, size=triples, p=weights / weights.sum())]
    trip = np.stack([subjects, rng.integers(0, relations, size=triples), rng.integers(0, entities, size=triples)], axis=1)
    sitelinks = rng.integers(0, 50, size=entities)
    prose = [" ".join(_words(rng, 10, syllables=(1, 3), capital=False).tolist()) for _ in range(2000)]
    return World(ents, rels, trip.astype(np.int64), sitelinks, prose)


class PairIndex:
    """The world's distinct (subject, relation) pairs with their object positions, held as
    sorted numpy arrays (a 10 M-triple world needs no Python set per pair)."""

    def __init__(self, triples: np.ndarray, relations: int) -> None:
        t = np.asarray(triples, dtype=np.int64).reshape(-1, 3)
        t = t[np.lexsort((t[:, 2], t[:, 1], t[:, 0]))]
        self._relations = max(int(relations), 1)
        key = t[:, 0] * self._relations + t[:, 1]
        self.keys, self._starts = np.unique(key, return_index=True)
        self._ends = np.append(self._starts[1:], len(key))
        self._objects = t[:, 2]

    def __len__(self) -> int:
        return len(self.keys)

    def random_pair(self, rng: np.random.Generator) -> tuple[int, int]:
        key = int(self.keys[int(rng.integers(len(self.keys)))])
        return key // self._relations, key % self._relations

    def items(self):
        """((subject, relation), objects) of every pair, in (subject, relation) order."""
        for k, key in enumerate(self.keys.tolist()):
            yield (key // self._relations, key % self._relations), set(
                self._objects[self._starts[k]: self._ends[k]].tolist())

    def objects(self, pair: tuple[int, int]) -> set[int]:
        key = pair[0] * self._relations + pair[1]
        at = int(np.searchsorted(self.keys, key))
        if at == len(self.keys) or int(self.keys[at]) != key:
            return set()
        return set(self._objects[self._starts[at]: self._ends[at]].tolist())


def object_sets(world: World) -> PairIndex:
    """The world's (subject, relation) pairs with their object positions."""
    return PairIndex(world.triples, len(world.relations))


def request_edits(world: World, pairs: PairIndex, rng: np.random.Generator,
                  count: int) -> list[tuple[str, str, str | None]]:
    """`count` seeded add/remove-triple edits of one request, written as the reference's
    pair-replacement edits (src/xgraph/kgversions.py:203-216): adding o to the pair (s, r)
    writes the pair's objects with o, removing o writes them without it (the pair deleted,
    object None, when none remain); one request's edits to a pair accumulate.  Half the
    edits touch pairs the world has (removing one of their objects, or adding one)."""
    entities, relations = len(world.entities), len(world.relations)
    changed: dict[tuple[int, int], set[int]] = {}
    for _ in range(count):
        if len(pairs) and rng.random() < 0.5:
            pair = pairs.random_pair(rng)
        else:
            pair = (int(rng.integers(entities)), int(rng.integers(relations)))
        objects = changed.setdefault(pair, pairs.objects(pair))
        if objects and rng.random() < 0.5:
            objects.discard(sorted(objects)[int(rng.integers(len(objects)))])
        else:
            objects.add(int(rng.integers(entities)))
    edits: list[tuple[str, str, str | None]] = []
    for (s, r), objects in changed.items():
        sid, rid = world.entities[s][0], world.relations[r][0]
        if objects:
            edits.extend((sid, rid, world.entities[o][0]) for o in sorted(objects))
        else:
            edits.append((sid, rid, None))
    return edits


def synthetic_tokenizer(world: World, vocab_size: int, syntax, seed: int = 0):
    """A byte-level BPE with exactly vocab_size ids (special <|endoftext|> included):
    the 256 byte tokens alone when vocab_size <= 257, else trained on the labels, the
    prose and the span delimiters, then padded with non-special added tokens."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers

    from .tokenizer import ServedTokenizer

    alphabet = sorted(pre_tokenizers.ByteLevel.alphabet())
    if vocab_size <= 257:
        tok = Tokenizer(models.BPE({c: i for i, c in enumerate(alphabet)}, []))
        tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
        tok.decoder = decoders.ByteLevel()
        if vocab_size == 257:
            tok.add_special_tokens(["<|endoftext|>"])
        return ServedTokenizer(tok)
    corpus = [syntax.label_prefix + label for _, labels in world.entities + world.relations for label in labels]
    corpus += world.prose
    spans = [syntax.opener + syntax.label_prefix + "x" + syntax.separator + syntax.label_prefix + "y" + syntax.closer,
             syntax.opener + syntax.escape + " x" + syntax.closer]
    corpus += spans * 200
    tok = Tokenizer(models.BPE())
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=vocab_size, special_tokens=["<|endoftext|>"],
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False)
    tok.train_from_iterator(corpus, trainer=trainer)
    short = vocab_size - tok.get_vocab_size(with_added_tokens=True)
    if short > 0:
        tok.add_tokens([f"<pad_{k}>" for k in range(short)])
    served = ServedTokenizer(tok)
    if served.vocab_size != vocab_size:
        raise RuntimeError(f"tokenizer has {served.vocab_size} ids, wanted {vocab_size}")
    return served


@dataclass(frozen=True)
class Config:
    name: str
    entities: int
    relations: int
    triples: int
    vocab: int
    rows: int
    lengths: tuple[int, int]
    labels: tuple[int, int] = (1, 1)
    zipf: float | None = None
    options: dict = field(default_factory=dict)
    dtype: str = "bfloat16"
    # continuous batching (the versions configuration): requests per second over the whole
    # job, the GPUs it is spread over, the simulated decode step, the geometric mean output
    # length and the most seeded edits (a private KG version) per request
    arrivals: float | None = None
    gpus: int = 1
    step_ms: float = 0.0
    mean_length: float = 0.0
    max_edits: int = 0


CONFIGS = {
    1: Config("toy-1k", 1_000, 20, 5_000, 256, 16, (64, 64), dtype="float32"),
    2: Config("ordinary-20k", 20_000, 50, 100_000, 32_000, 64, (256, 256), dtype="float32"),
    3: Config("paths-100k", 100_000, 100, 1_000_000, 128_256, 256, (64, 1024), labels=(1, 3),
              options={"paths": True, "committed_paths": True}),
    4: Config("paths-1m-zipf", 1_000_000, 200, 10_000_000, 128_256, 512, (64, 1024), zipf=1.1,
              options={"paths": True, "committed_paths": True}),
    # 2,000 requests/s over 8 GPUs, one decode step every 2 ms: 0.5 arrivals per step per
    # GPU against 128 rows whose requests last 256 steps on average, so the live batch
    # hovers at its 128-row cap (1,024 over the 8 GPUs)
    5: Config("versions-1m", 1_000_000, 200, 10_000_000, 151_936, 128, (1, 1024), zipf=1.1,
              options={"paths": True, "committed_paths": True}, arrivals=2000.0, gpus=8, step_ms=2.0,
              mean_length=256.0, max_edits=256),
}


@dataclass
class Arrivals:
    """A continuous-batching replay on one GPU: per request its arrival step, output length
    and (once admitted) slot and first step; per step the requests admitted (slot, request)
    and the slots live in it, in slot order."""

    arrival: list[int]
    length: list[int]
    slot: list[int]
    start: list[int]
    admitted: list[list[tuple[int, int]]]
    live: list[list[int]]


def arrival_schedule(config: Config, steps: int, seed: int, rank: int = 0, *, max_length: int | None = None) -> Arrivals:
    """Poisson arrivals at config.arrivals / config.gpus requests per second on a clock of
    one step every config.step_ms, output lengths Geometric(mean config.mean_length) (capped
    at max_length, default the configuration's longest), served first come first served in
    config.rows slots: a request leaves its slot after its last token and a waiting request
    takes it at the next step.  The batch starts full (the geometric length is memoryless,
    so the requests live at step 0 are as long as any), and the steps' batches are ragged."""
    rng = np.random.default_rng(seed * 1009 + rank)
    cap = max_length or config.lengths[1]
    rate = config.arrivals / config.gpus * config.step_ms / 1000.0
    counts = np.concatenate([[config.rows], rng.poisson(rate, size=steps - 1)]) if steps else np.zeros(0, int)
    arrival = np.repeat(np.arange(steps), counts).tolist()
    length = np.minimum(rng.geometric(1.0 / config.mean_length, size=len(arrival)), cap).tolist()
    slot, start = [-1] * len(arrival), [-1] * len(arrival)
    free = list(range(config.rows - 1, -1, -1))
    ends: dict[int, list[int]] = {}
    waiting, admitted, live, nxt = [], [], [], 0
    occupant: dict[int, int] = {}
    for k in range(steps):
        for s in ends.pop(k, []):
            del occupant[s]
            free.append(s)
        free.sort(reverse=True)
        while nxt < len(arrival) and arrival[nxt] <= k:
            waiting.append(nxt)
            nxt += 1
        joined = []
        while waiting and free:
            r, s = waiting.pop(0), free.pop()
            slot[r], start[r] = s, k
            occupant[s] = r
            ends.setdefault(k + length[r], []).append(s)
            joined.append((s, r))
        admitted.append(joined)
        live.append(sorted(occupant))
    return Arrivals(arrival, length, slot, start, admitted, live)


@dataclass
class Workload:
    config: Config
    world: World
    served: object
    syntax: object
    index: object


def build_workload(number: int, seed: int | None = None, device=None) -> Workload:
    """Config `number`'s world, served tokenizer and KG index (seeded by `seed`, default
    the config number); `device` builds the index's edge arrays on that GPU."""
    from .index import build_kg_index_arrays
    from .syntax import SpanSyntax

    config = CONFIGS[number]
    syntax = SpanSyntax()
    world = synthetic_world(number if seed is None else seed, config.entities, config.relations, config.triples,
                            labels=config.labels, zipf=config.zipf)
    served = synthetic_tokenizer(world, config.vocab, syntax)
    index = build_kg_index_arrays(world.entities, world.relations, world.triples, served, syntax,
                                  sitelinks=world.sitelinks, device=device)
    return Workload(config, world, served, syntax, index)


# ---------------------------------------------------------------------------------------
# Constrained stream sampling on the GPU.

def _delimiter_like(served, syntax) -> np.ndarray:
    delims = [d.encode("utf-8") for d in (syntax.closer, syntax.separator, syntax.escape)]
    out = np.zeros(served.vocab_size, dtype=bool)
    for t in range(served.vocab_size):
        b = served.token_bytes(t)
        if b and any(d.find(b) >= 0 for d in delims):
            out[t] = True
    return out


def _prose_tokens(served, world: World) -> np.ndarray:
    out = np.zeros(served.vocab_size, dtype=bool)
    for line in world.prose[:400]:
        out[served.encode(" " + line)] = True
    return out


def sample_streams(engine, served, syntax, world: World, rows: int, steps: int, seed: int,
                   *, p_open=0.25, p_sep=0.5, p_close=0.8, p_escape=0.05, p_unescape=0.3, record=None,
                   device: str = "cuda", versions=None):
    """Constrained random walks of `rows` slots for `steps` tokens, decoded on the GPU with
    the engine as the constraint.  Returns (tokens [rows, steps] int32 on the GPU, allowed
    counts [rows, steps + 1] int32: how many ids each step's mask allowed).  `record`
    (optional set of (row, step)) collects those masks on the host for parity checks;
    `versions` (optional, one KG version name or None per row) pins each row's version."""
    import torch

    device = torch.device(device)
    gen = torch.Generator(device=device).manual_seed(seed)
    vocab, words = served.vocab_size, engine.words
    queues = [served.encode(" " + syntax.opener), served.encode(syntax.separator),
              served.encode(syntax.closer), served.encode(syntax.escape)]
    qlen = torch.tensor([len(q) for q in queues], device=device)
    qtok = torch.zeros((4, max(len(q) for q in queues)), dtype=torch.long, device=device)
    for k, q in enumerate(queues):
        qtok[k, : len(q)] = torch.tensor(q)
    special = torch.zeros(vocab, dtype=torch.bool, device=device)
    special[list(served.special_ids)] = True
    label_like = ~torch.from_numpy(_delimiter_like(served, syntax)).to(device) & ~special
    prose = torch.from_numpy(_prose_tokens(served, world)).to(device)
    engine.reset()
    slots = torch.arange(rows, dtype=torch.int32, device=device)
    engine.begin(slots)
    for row, name in enumerate(versions or ()):
        engine.set_version(row, name)
    kind = torch.full((rows,), -1, dtype=torch.long, device=device)
    pos = torch.zeros(rows, dtype=torch.long, device=device)
    tokens = torch.zeros((rows, steps), dtype=torch.int32, device=device)
    counts = torch.zeros((rows, steps + 1), dtype=torch.int32, device=device)
    shifts = torch.arange(32, device=device, dtype=torch.int32)
    masks = engine.mask_view()
    states = engine.states_view()
    recorded = {}
    for step in range(steps + 1):
        engine.fill_mask(rows)
        bits = ((masks[:rows].unsqueeze(-1) >> shifts) & 1).bool().reshape(rows, -1)[:, :vocab]
        counts[:, step] = bits.sum(1, dtype=torch.int32)
        if record:
            for r, s in record:
                if s == step:
                    recorded[(r, s)] = masks[r, :words].clone()
        if step == steps:
            break
        phase = states[:rows, 0].long()
        u = torch.rand((rows, 3), generator=gen, device=device)
        idle = kind < 0
        can_sep = bits[:, queues[1][0]]
        can_close = bits[:, queues[2][0]]
        start = torch.full_like(kind, -1)
        start = torch.where(idle & (phase == 0) & (u[:, 0] < p_open), 0, start)
        span = idle & (phase == 1)
        start = torch.where(span & can_sep & (u[:, 0] < p_sep), 1, start)
        start = torch.where(span & (start < 0) & can_close & (u[:, 1] < p_close), 2, start)
        start = torch.where(span & (start < 0) & (u[:, 2] < p_escape), 3, start)
        start = torch.where(idle & (phase == 2) & (u[:, 0] < p_unescape), 2, start)
        kind = torch.where(start >= 0, start, kind)
        pos = torch.where(start >= 0, 0, pos)
        queued = qtok[kind.clamp(min=0), pos]
        take = (kind >= 0) & bits.gather(1, queued.unsqueeze(1)).squeeze(1)
        prefer = torch.where((phase == 1).unsqueeze(1), label_like.unsqueeze(0), prose.unsqueeze(0)) & bits
        prefer = torch.where(prefer.any(1, keepdim=True), prefer, bits & ~special.unsqueeze(0))
        prefer = torch.where(prefer.any(1, keepdim=True), prefer, bits)
        noise = torch.rand((rows, vocab), generator=gen, device=device)
        drawn = torch.where(prefer, noise, -1.0).argmax(1)
        choice = torch.where(take, queued, drawn)
        pos = torch.where(take, pos + 1, 0)
        kind = torch.where(take & (pos < qlen[kind.clamp(min=0)]), kind, -1)
        pos = torch.where(kind < 0, 0, pos)  # a finished or abandoned queue restarts at 0
        tokens[:, step] = choice.int()
        engine.advance(choice.int())
    if engine.errors(rows):
        raise RuntimeError("a sampled stream left the mask")
    return tokens, counts, {k: v.cpu().numpy().view(np.uint32) for k, v in recorded.items()}
