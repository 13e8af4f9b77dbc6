"""Token id -> bytes table (the vocabulary the automata consume).

Field-for-field compatible with bpdecode's ``Vocabulary``
(``src/bpdecode/tokenizer.py:27-92``): ``token_bytes`` (a tuple of ``bytes``)
and ``eos_id``. Any object with those two attributes is accepted wherever a
vocabulary is expected, so a vocabulary built by bpdecode itself (for example
with ``Vocabulary.from_hf``) drops in unchanged.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Vocabulary:
    """Token id -> UTF-8 bytes, plus the id that signals end-of-sequence."""

    token_bytes: tuple[bytes, ...]
    eos_id: int | None = None

    def __len__(self) -> int:
        return len(self.token_bytes)

    @property
    def size(self) -> int:
        return len(self.token_bytes)

    def decode(self, ids: list[int]) -> bytes:
        return b"".join(self.token_bytes[i] for i in ids)

    @classmethod
    def from_tokens(
        cls, tokens: list[str] | list[bytes], eos_id: int | None = None
    ) -> Vocabulary:
        tb = tuple(t if isinstance(t, bytes) else t.encode("utf-8") for t in tokens)
        return cls(token_bytes=tb, eos_id=eos_id)

    @classmethod
    def from_hf(cls, tokenizer_or_name: object) -> Vocabulary:
        """Delegate to bpdecode's Hugging Face loader (a compile-time front-end
        this package does not rebuild)."""
        try:
            from bpdecode.tokenizer import Vocabulary as _RefVocab  # type: ignore
        except ImportError as exc:  # pragma: no cover - optional front-end
            raise ImportError(
                "Vocabulary.from_hf needs the bpdecode front-end package installed"
            ) from exc
        v = _RefVocab.from_hf(tokenizer_or_name)
        return cls(token_bytes=tuple(v.token_bytes), eos_id=v.eos_id)


def as_vocabulary(obj: object) -> Vocabulary:
    """Accept this package's Vocabulary, any duck-typed equivalent, or a
    Hugging Face tokenizer."""
    if isinstance(obj, Vocabulary):
        return obj
    if hasattr(obj, "token_bytes"):
        return Vocabulary(tuple(obj.token_bytes), getattr(obj, "eos_id", None))
    return Vocabulary.from_hf(obj)
