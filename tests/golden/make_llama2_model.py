"""Seeded synthetic llama2 checkpoints and tokenizers in the format
benchmarks/llama2/llama.cpp reads (the llama2.c format).

The reference runs a trained checkpoint (llama2/Makefile:9, stories15M.bin)
that is not in its tree, so the tests and the benchmark use random weights of
a given shape instead:

* checkpoint (llama2/llama.cpp:150-169, 111-148): the 7 int32 Config fields
  (dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len;
  vocab_size < 0 = a separate classifier), then fp32 token_embedding_table,
  rms_att_weight, wq, wk, wv, wo, rms_ffn_weight, w1, w2, w3,
  rms_final_weight, seq_len * head_size of unused RoPE tables and, when
  not shared, the classifier wcls [vocab_size x dim];
* tokenizer (llama2/llama.cpp:411-436): int32 max_token_length, then per
  token fp32 score, int32 length, bytes.  Tokens: 0 <unk>, 1 BOS, 2 EOS,
  3..258 the byte tokens <0x00>..<0xFF>, then the printable ASCII
  characters (the encoder needs " " for its dummy prefix), then two-letter
  merges up to vocab_size.

    python tests/golden/make_llama2_model.py <out_dir> [--shape tiny|stories15M]
"""
from __future__ import annotations

import argparse
import os
import string
import struct

import numpy as np

# (dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len, shared classifier)
SHAPES = {
    # grouped-query attention (kv_dim = dim / 2) so the K/V rows differ from
    # Q's, and a separate classifier (with the shared one, random weights
    # mostly predict the input token back)
    "tiny": (128, 384, 2, 4, 2, 512, 64, False),
    # the reference's default model (llama2/Makefile:9, stories15M)
    "stories15M": (288, 768, 6, 6, 6, 32000, 256, True),
}


def write_checkpoint(path: str, shape: tuple, seed: int = 0) -> None:
    dim, hidden, layers, heads, kv_heads, vocab, seq_len, shared = shape
    head = dim // heads
    kv_dim = dim * kv_heads // heads
    rng = np.random.default_rng(seed)

    def normal(n, std):
        return (rng.standard_normal(n, dtype=np.float32) * np.float32(std)).astype(np.float32)

    parts = [
        normal(vocab * dim, 1.0),                      # token_embedding_table
        1.0 + normal(layers * dim, 0.1),               # rms_att_weight
        normal(layers * dim * dim, dim ** -0.5),       # wq
        normal(layers * dim * kv_dim, dim ** -0.5),    # wk
        normal(layers * dim * kv_dim, dim ** -0.5),    # wv
        normal(layers * dim * dim, dim ** -0.5),       # wo
        1.0 + normal(layers * dim, 0.1),               # rms_ffn_weight
        normal(layers * dim * hidden, dim ** -0.5),    # w1
        normal(layers * hidden * dim, hidden ** -0.5),  # w2
        normal(layers * dim * hidden, dim ** -0.5),    # w3
        1.0 + normal(dim, 0.1),                        # rms_final_weight
        np.zeros(seq_len * head, np.float32),          # unused RoPE tables
    ]
    if not shared:
        parts.append(normal(vocab * dim, dim ** -0.5))  # wcls
    with open(path, "wb") as f:
        f.write(struct.pack("7i", dim, hidden, layers, heads, kv_heads, vocab if shared else -vocab, seq_len))
        for p in parts:
            f.write(p.tobytes())


def vocab_pieces(vocab: int) -> list[bytes]:
    pieces = [b"<unk>", b"\n<s>\n", b"\n</s>\n"]
    pieces += [f"<0x{i:02X}>".encode() for i in range(256)]
    pieces += [c.encode() for c in string.printable[:95]]  # digits, letters, punctuation, space
    letters = string.ascii_lowercase
    merges = [(" " + a).encode() for a in letters] + [(a + b).encode() for a in letters for b in letters]
    pieces += merges[: max(0, vocab - len(pieces))]
    if len(pieces) < vocab:
        pieces += [f"<extra{i}>".encode() for i in range(vocab - len(pieces))]
    return pieces[:vocab]


def write_tokenizer(path: str, vocab: int) -> None:
    pieces = vocab_pieces(vocab)
    with open(path, "wb") as f:
        f.write(struct.pack("i", max(len(p) for p in pieces)))
        for i, p in enumerate(pieces):
            score = -float(i) if i >= 259 + 95 else 0.0  # earlier merges win
            f.write(struct.pack("fi", score, len(p)))
            f.write(p)


def write_model(out_dir: str, shape: str = "tiny", seed: int = 0) -> tuple[str, str]:
    os.makedirs(out_dir, exist_ok=True)
    ckpt = os.path.join(out_dir, f"{shape}.bin")
    tok = os.path.join(out_dir, f"{shape}_tokenizer.bin")
    write_checkpoint(ckpt, SHAPES[shape], seed)
    write_tokenizer(tok, SHAPES[shape][5])
    return ckpt, tok


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("out_dir")
    ap.add_argument("--shape", default="tiny", choices=sorted(SHAPES))
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    for p in write_model(a.out_dir, a.shape, a.seed):
        print(p)
