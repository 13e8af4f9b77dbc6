"""Context-free grammar path: :mod:`bpdecode_b200.grammar.device`."""
