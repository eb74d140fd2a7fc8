"""Generate tests/golden/*.npz from the reference's own CPU backend.

Run in a checkout where oracle/_ref/libomni_ref_cpu.so was built from the
reference sources (`make -C oracle ref`):

    python tests/golden/make_golden.py

Every fixture stores the inputs and the reference's output, so the oracle
(oracle/omni_oracle.c) can be pinned on machines without the reference.
Inputs use the deterministic LCG of the reference's native tests or seeded
numpy draws; nothing here is copied from the reference's test data.
"""

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent

ATTENTION = [
    # name, rows, heads, hd, block, valid, fused, bf16
    ("attn_ref_odd", 17, 3, 7, 5, 11, False, False),
    ("attn_ref_fused_bf16", 33, 3, 11, 0, 33, True, True),
    ("attn_block_valid_hd64", 257, 2, 64, 200, 205, False, False),
    ("attn_bf16_hd64", 160, 2, 64, 0, 160, False, True),
    ("attn_bf16_hd72", 140, 2, 72, 0, 140, False, True),
    ("attn_fused_bf16_hd96", 150, 2, 96, 0, 150, True, True),
    ("attn_keypad_hd64", 300, 2, 64, 0, 217, False, True),
]

# Head-major batched attention (oracle.attention_bhld): name, batch, heads, L, hd, lengths, block.
ATTENTION_BHLD = [
    ("attn_bhld_varlen_hd64", 3, 2, 100, 64, (100, 67, 1), 0),
    ("attn_bhld_block_hd72", 2, 2, 90, 72, (90, 83), 40),
]


def bhld_fixtures():
    """Each (batch, head) slice of a head-major batch is the reference's
    Ops::attention on one sequence of `heads=1`, valid = lengths[b]."""
    assert O.ref_available(), "build oracle/_ref first: make -C oracle ref"
    for name, batch, heads, L, hd, lengths, block in ATTENTION_BHLD:
        shape = (batch, heads, L, hd)
        q = O.lcg_values(int(np.prod(shape)), 321).reshape(shape)
        k = O.lcg_values(int(np.prod(shape)), 654).reshape(shape)
        v = O.lcg_values(int(np.prod(shape)), 987).reshape(shape)
        y = np.zeros(shape, np.float32)
        for b in range(batch):
            for h in range(heads):
                y[b, h] = O.attention(q[b, h], k[b, h], v[b, h], 1, block, lengths[b], impl="ref")
        np.savez_compressed(OUT / f"{name}.npz", kind="attention_bhld", q=q, k=k, v=v, y=y,
                            lengths=np.array(lengths, np.int32), block=block)


def main():
    assert O.ref_available(), "build oracle/_ref first: make -C oracle ref"
    bhld_fixtures()
    for name, rows, heads, hd, block, valid, fused, bf16 in ATTENTION:
        d = heads * hd
        cols = d * (3 if fused else 1)
        q = O.lcg_values(rows * cols, 123).reshape(rows, cols)
        k = O.lcg_values(rows * d, 456).reshape(rows, d)
        v = O.lcg_values(rows * d, 789).reshape(rows, d)
        y = O.attention(q, k, v, heads, block, valid, fused, bf16, impl="ref")
        np.savez_compressed(OUT / f"{name}.npz", kind="attention", q=q, k=k, v=v, y=y, heads=heads,
                            block=block, valid=valid, fused=fused, bf16=bf16)
    rng = np.random.default_rng(2024)
    for name, rows, dim, codes, bf16 in [
        ("vq_bf16_d32", 200, 32, 1500, True),
        ("vq_bf16_d64", 150, 64, 1300, True),
        ("vq_fp32_d64", 120, 64, 1030, False),
    ]:
        x = rng.standard_normal((rows, dim)).astype(np.float32)
        cb = rng.standard_normal((codes, dim)).astype(np.float32)
        if bf16:
            x, cb = O.round_bf16(x), O.round_bf16(cb)
        cb[5] = x[0]
        cb[1027] = x[0]  # duplicate winner across the 1024/256 tile boundaries
        cbnorm = O.squares(cb, bf16=bf16, impl="ref")
        ids = O.quantize(x, cb, cbnorm, bf16=bf16, impl="ref")
        np.savez_compressed(OUT / f"{name}.npz", kind="quantize", x=x, cb=cb, cbnorm=cbnorm, ids=ids, bf16=bf16)
    x = O.lcg_values(40 * 48, 7).reshape(40, 48) * 4
    for bf16 in (False, True):
        y = O.squares(x, bf16=bf16, impl="ref")
        np.savez_compressed(OUT / f"squares_{'bf16' if bf16 else 'fp32'}.npz", kind="squares", x=x, y=y, bf16=bf16)
    print("wrote", len(list(OUT.glob("*.npz"))), "fixtures to", OUT)


if __name__ == "__main__":
    main()
