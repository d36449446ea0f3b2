"""The reference's own dense backend as the C4 oracle (CPU, no GPU needed).

oracle/_ref/katali_dropin is the reference's gguf_model.c / katali_dense_cuda.c and the files
they need, compiled unchanged, with this repository's katali_cuda.h and dlopen loader in place
of the reference's missing src/katali_cuda.c. With KATALI_CUDA=0 it decodes on the
reference's CPU path (gguf_forward_token, V/src/gguf_model.c:570-703). This checks that the
step composed from the reference's kernels (oracle.RefDense, the oracle of the GPU dense
decoder tests) gives bit-identical logits at every step and the same greedy tokens, so that
oracle is the reference's forward pass itself."""
import os

import numpy as np
import pytest

from oracle.oracle import DROPIN, RefDense, rel_l2
from tests.dropin_util import N_TOKENS, host_model, prompt_ids, run_reference, write_model

pytestmark = pytest.mark.skipif(not os.path.exists(DROPIN),
                                reason="the reference's dense backend was not built (no reference checkout)")


def test_reference_forward_matches_composed_oracle(ref, port, tmp_path):
    data, offsets = write_model(port, tmp_path / "m.gguf")
    rec, lg, ids = run_reference(tmp_path / "m.gguf", tmp_path / "cpu", cuda=False)
    assert rec["cuda_enabled"] == 0 and rec["generated"] == N_TOKENS == rec["observed"]
    rd = RefDense(ref, host_model(data, offsets))
    seq = prompt_ids()
    for s, t in enumerate(seq[:-1]):
        rd.step(t, s)
    pos, tok = len(seq) - 1, seq[-1]
    for i in range(N_TOKENS):
        lc = rd.step(tok, pos)
        assert np.array_equal(lg[i], lc), (i, rel_l2(lg[i], lc))
        tok = port.argmax(lc)
        assert tok == int(ids[i]), i
        pos += 1
    rd.close()
