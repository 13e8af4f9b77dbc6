"""Seeded synthetic workloads for the benchmark configurations.

No real tokenizer or model weights are available offline, so every
configuration runs on a synthetic vocabulary drawn from a fixed seed. The
shapes and value distributions follow the benchmark configurations of the
constrained-decoding step:

* config 1 -- V = 32,000; byte length uniform 1..8; each byte 70% from
  ``[0-9.a-zA-Z ]`` and 30% uniform in 0x21..0x7E; id 31999 is ``<eos>``.
* configs 2, 4, 5 (V = 128,256) and 3 (V = 151,936) -- byte length
  geometric(p = 0.3) capped at 16; each character 85% printable ASCII
  0x20..0x7E, 15% a valid 2..4-byte UTF-8 scalar (no surrogates), never
  splitting a character; a single ``<eos>`` at V - 1; the single-byte tokens
  ``{ [ " , } ] :`` reserved at ids 0..6 so the config-4 logit bias has targets.

Everything is a pure function of the seed, so every GPU rank, the CPU oracle
and the test fixtures see identical vocabularies.
"""

from __future__ import annotations

import random
from dataclasses import dataclass

from .tokenizer import Vocabulary

# The eight regexes of the serving-scale dense configuration (one per row,
# chosen uniformly from the seed).
DENSE_PATTERNS: tuple[tuple[str, str], ...] = (
    ("ipv4", r"([0-9]{1,3}\.){3}[0-9]{1,3}"),
    ("date", r"\d{4}-\d{2}-\d{2}"),
    ("email", r"[a-z0-9._]+@[a-z]+\.[a-z]{2,4}"),
    ("float", r"[+-]?[0-9]+\.[0-9]+([eE][+-]?[0-9]+)?"),
    ("hexcolour", r"#[0-9a-fA-F]{6}"),
    ("uuid", r"[0-9a-f]{8}-[0-9a-f]{4}-[0-9a-f]{4}-[0-9a-f]{4}-[0-9a-f]{12}"),
    ("name", r"[A-Z][a-z]{2,15}( [A-Z][a-z]{2,15}){0,3}"),
    ("phone", r"\+?[0-9]{1,3}[ -]?\(?[0-9]{3}\)?[ -]?[0-9]{3}[ -]?[0-9]{4}"),
)

IPV4_PATTERN = DENSE_PATTERNS[0][1]

# The non-recursive JSON-Schema object of config 3. The 6-value enum set is
# not fixed by the configuration text; this one is.
TAG_ENUM = ("alpha", "beta", "gamma", "delta", "epsilon", "zeta")
SCHEMA_OBJECT = {
    "type": "object",
    "properties": {
        "id": {"type": "integer"},
        "name": {"type": "string", "maxLength": 24},
        "score": {"type": "number"},
        "tags": {"type": "array", "items": {"enum": list(TAG_ENUM)}, "maxItems": 4},
        "active": {"type": "boolean"},
    },
    "required": ["id", "name", "score", "tags", "active"],
    "additionalProperties": False,
}

# Reserved single-byte tokens at ids 0..6 of the large vocabularies.
RESERVED = (b"{", b"[", b'"', b",", b"}", b"]", b":")
BIASED = (b"{", b"[", b'"', b",")  # +3 logit bias in the recursive-GBNF config
OPENERS = (b"(", b"[")  # +1 logit bias in the brackets (memo-miss) workload


def token_ids(vocab, tokens) -> list[int]:
    """Every id whose bytes equal one of `tokens` (a synthetic vocabulary may
    hold a byte string more than once)."""
    want = set(tokens)
    return [i for i, t in enumerate(vocab.token_bytes) if t in want]

_CONFIG1_ALPHABET = b"0123456789.abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ "


def vocab_config1(seed: int = 0, size: int = 32_000) -> Vocabulary:
    """Config-1 vocabulary: lengths uniform 1..8, 70% regex-friendly bytes."""
    rng = random.Random(seed)
    out: list[bytes] = []
    for _ in range(size - 1):
        n = rng.randint(1, 8)
        tok = bytearray()
        for _ in range(n):
            if rng.random() < 0.7:
                tok.append(_CONFIG1_ALPHABET[rng.randrange(len(_CONFIG1_ALPHABET))])
            else:
                tok.append(rng.randint(0x21, 0x7E))
        out.append(bytes(tok))
    out.append(b"<eos>")
    return Vocabulary(tuple(out), eos_id=size - 1)


def _utf8_scalar(rng: random.Random) -> bytes:
    nbytes = rng.choice((2, 3, 4))
    if nbytes == 2:
        cp = rng.randint(0x80, 0x7FF)
    elif nbytes == 3:
        while True:
            cp = rng.randint(0x800, 0xFFFF)
            if not 0xD800 <= cp <= 0xDFFF:
                break
    else:
        cp = rng.randint(0x10000, 0x10FFFF)
    return chr(cp).encode("utf-8")


def _geometric(rng: random.Random, p: float, cap: int) -> int:
    n = 1
    while n < cap and rng.random() >= p:
        n += 1
    return n


def vocab_large(size: int = 128_256, seed: int = 0) -> Vocabulary:
    """Configs 2-5 vocabulary (see module docstring)."""
    rng = random.Random(seed * 7919 + size)
    out: list[bytes] = list(RESERVED)
    for _ in range(size - 1 - len(RESERVED)):
        budget = _geometric(rng, 0.3, 16)
        tok = bytearray()
        while len(tok) < budget:
            if rng.random() < 0.85:
                ch = bytes((rng.randint(0x20, 0x7E),))
            else:
                ch = _utf8_scalar(rng)
                if len(tok) + len(ch) > budget:
                    if tok:
                        break
                    ch = bytes((rng.randint(0x20, 0x7E),))
            tok += ch
        out.append(bytes(tok))
    out.append(b"</s>")
    return Vocabulary(tuple(out), eos_id=size - 1)


def row_patterns(batch: int, seed: int = 0, n_patterns: int = len(DENSE_PATTERNS)) -> list[int]:
    """Pattern index per row, uniform from the seed (config 2)."""
    rng = random.Random(seed * 104729 + batch)
    return [rng.randrange(n_patterns) for _ in range(batch)]


# Global row blocks of the serving-scale dense configuration. The request
# rows of a multi-GPU run are numbered globally and cut into blocks of
# ROW_BLOCK rows; everything random about a row (its pattern, its logits at
# every step) is a function of its block and its position in the block only,
# so a rank that owns block b computes exactly what one process running the
# whole global batch computes for those rows.
ROW_BLOCK = 1024


def block_patterns(block: int, rows: int = ROW_BLOCK) -> list[int]:
    """Pattern index of each row of global row block ``block``."""
    return row_patterns(rows, seed=block)


def block_logits_seed(block: int, step: int) -> int:
    """Seed of the logits of global row block ``block`` at generation step
    ``step`` (a torch.Generator on the row block's device)."""
    return block * 1_000_003 + step


@dataclass(frozen=True)
class DenseConfig:
    name: str
    vocab_size: int
    batch: int
    dtype: str  # "fp32" | "bf16"
    sigma: float
    steps: int


CONFIG1 = DenseConfig("config1-ipv4-v32000-b64-fp32", 32_000, 64, "fp32", 1.0, 32)
CONFIG2 = DenseConfig("config2-8regex-v128256-b1024-bf16", 128_256, 1024, "bf16", 2.0, 128)
CONFIG3 = DenseConfig("config3-jsonschema-v151936-b512-fp32", 151_936, 512, "fp32", 1.0, 256)
