"""Caption tokenisation into the fixed-width rows the text encoders take.

Row layouts (the reference's, prepare_data.py / sample_ckpt.py:32-41):
  from-scratch encoder: [BOS] ids[: max - 2] [EOS] PAD..., PAD = 0, BOS 2, EOS 3, NULL prompt = [BOS, NULL, EOS]
  frozen-LM encoders  : [BOS] ids[: max - 1] PAD..., PAD = 65535 (the LM's own BOS id)
A local ``tokenizer.json`` (HF ``tokenizers``) is used when given; ``ByteTokenizer`` is a dependency-free stand-in
(UTF-8 bytes shifted past the special ids) for smoke runs and tests.
"""
import numpy as np
import torch

PAD_ID, BOS_ID, EOS_ID = 0, 2, 3
LM_PAD = 65535


class ByteTokenizer:
    def __init__(self, vocab=8192, offset=6):
        self.vocab, self.offset = vocab, offset

    def encode(self, text):
        return [min(self.vocab - 1, b + self.offset) for b in " ".join(text.split()).encode("utf-8")]


class FileTokenizer:
    def __init__(self, path):
        from tokenizers import Tokenizer
        self.tok = Tokenizer.from_file(path)

    def encode(self, text):
        return self.tok.encode(" ".join(text.split()), add_special_tokens=False).ids


def load_tokenizer(path=None, vocab=8192):
    return FileTokenizer(path) if path else ByteTokenizer(vocab)


def tokenize(texts, max_tokens, tokenizer, lm=False, bos=None):
    if lm:
        rows = np.full((len(texts), max_tokens), LM_PAD, dtype=np.int64)
        for i, t in enumerate(texts):
            ids = tokenizer.encode(t)[: max_tokens - 1]
            rows[i, 0] = BOS_ID if bos is None else bos
            rows[i, 1:1 + len(ids)] = ids
    else:
        rows = np.full((len(texts), max_tokens), PAD_ID, dtype=np.int64)
        for i, t in enumerate(texts):
            ids = tokenizer.encode(t)[: max_tokens - 2]
            rows[i, 0] = BOS_ID
            rows[i, 1:1 + len(ids)] = ids
            rows[i, 1 + len(ids)] = EOS_ID
    return torch.from_numpy(rows)
