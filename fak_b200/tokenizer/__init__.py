"""Tokenizers: byte-level BPE from GGUF metadata or tokenizer.json, plus incremental detokenization."""
from .bpe import IncrementalDecoder, Tokenizer, bytes_to_unicode

__all__ = ["IncrementalDecoder", "Tokenizer", "bytes_to_unicode"]
