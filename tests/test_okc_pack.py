"""The restated host side of the reference operator (oracle/okc_ref.py) against the reference's own packers.

``oracle/okc_ref.py`` rebuilds, in torch, the layouts the reference's ``prepare`` writes (moe_w4a16.py:3168-3209
with the GF(2) word transform of :3903-3933) so that the reference's prebuilt kernel can run where its Python
is absent.  Here the rebuilt bytes must equal, digest for digest, what the reference's own functions produced on
the same seeded inputs (``tests/golden/ref_okc_pack.json``, made by ``tests/golden/make_golden.py``)."""
import hashlib
import json
import os

import numpy as np
import torch

from oracle import okc_ref
from tests.golden.make_golden import okc_pack_inputs

HERE = os.path.dirname(os.path.abspath(__file__))


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(np.ascontiguousarray(t.cpu().numpy()).tobytes()).hexdigest()


def test_restated_packers_equal_the_reference_packers():
    with open(os.path.join(HERE, "golden", "ref_okc_pack.json")) as f:
        want = json.load(f)
    c13, s13, c2, s2 = (torch.from_numpy(a) for a in okc_pack_inputs())
    cols = okc_ref._xc_cols()
    for tag, codes, sf, rows in (("gate_up", c13 ^ 0x88, s13, okc_ref.gate_up_rows(128)),
                                 ("down", c2, s2, torch.arange(256))):
        words = okc_ref.pack_code_words(codes, rows, cols)
        scales = okc_ref.pack_scale_bytes(sf, rows)
        assert [int(v) for v in words[:8]] == want[tag]["words_head"], tag
        assert _sha(words) == want[tag]["words"], tag
        assert _sha(scales) == want[tag]["scales"], tag
        assert _sha(okc_ref.fat_order(words, scales)) == want[tag]["fat"], tag
        assert _sha(okc_ref.unit_order(words, scales)) == want[tag]["unit"], tag
    assert _sha(okc_ref.e4m3_lut("cpu")) == want["lut"]


def test_build_choice_follows_the_reference_token_bounds():
    """M = 1: the program build; <= 4 TINY; <= 8 TINY2; <= 16 MID; above: the mma.sync MAIN build."""
    assert [okc_ref.build_for(m) for m in (1, 2, 4, 5, 8, 9, 16, 17, 32, 128, 256, 384, 1000)] == \
        ["program", "tiny", "tiny", "tiny2", "tiny2", "mid", "mid", "main", "main", "main", "main", "main", "main"]
