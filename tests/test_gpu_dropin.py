"""The drop-in, shown with the reference's own caller: its dense backend (gguf_model.c,
katali_dense_cuda.c, compiled unchanged; V/src/katali_dense_cuda.c:14-73 and
V/src/gguf_model.c:495-555 route every qwen3 projection to katali_cuda_matvec) runs a greedy
generate with KATALI_CUDA=1 through this repository's loader and plugin, and with
KATALI_CUDA=0 on its CPU path.

Bars: the reference switched its CUDA path on and every plugin matvec it called succeeded;
the logits it sampled from are within rel_L2 <= 1e-5 of its CPU run at every step and the
greedy tokens are identical. The on-device dense decoder built from the same file
(katali_cuda_dense_create_from_gguf) meets the same bars against the reference's CPU
forward pass."""
import os

import numpy as np
import pytest

from katali_lab_b200 import DenseModel, Gguf
from katali_lab_b200.build import PLUGIN
from oracle.oracle import DROPIN, rel_l2
from tests.dropin_util import CFG, N_TOKENS, prompt_ids, run_reference, write_model

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(DROPIN),
                                 reason="the reference's dense backend was not built")]


def test_reference_caller_through_the_plugin(plugin, port, tmp_path):
    write_model(port, tmp_path / "m.gguf")
    cpu, lc, ic = run_reference(tmp_path / "m.gguf", tmp_path / "cpu", cuda=False)
    gpu, lg, ig = run_reference(tmp_path / "m.gguf", tmp_path / "gpu", cuda=True, plugin_path=PLUGIN)
    assert gpu["cuda_enabled"] == 1, gpu
    # 7 projections per layer and the LM head per token, each one plugin matvec
    assert gpu["plugin_matvec_calls"] > 0 and gpu["plugin_matvec_ok"] == gpu["plugin_matvec_calls"], gpu
    assert cpu["plugin_matvec_calls"] == 0
    assert gpu["generated"] == cpu["generated"] == N_TOKENS
    for i in range(N_TOKENS):
        assert rel_l2(lg[i], lc[i]) <= 1e-5, (i, rel_l2(lg[i], lc[i]))
    assert ig.tolist() == ic.tolist()


def test_device_decoder_matches_reference_forward(plugin, port, tmp_path):
    write_model(port, tmp_path / "m.gguf")
    _, lc, ic = run_reference(tmp_path / "m.gguf", tmp_path / "cpu", cuda=False)
    g = Gguf(plugin, str(tmp_path / "m.gguf"))
    dm = DenseModel.from_gguf(plugin, g, kv_cap=CFG.kv_cap)
    g.close()
    seq = prompt_ids()
    for t in seq[:-1]:
        dm.generate([t], 1)
    tok = seq[-1]
    for i in range(N_TOKENS):
        tok = int(dm.generate([tok], 1)[0])
        ptr, _ = dm.logits()
        lg = np.empty(CFG.vocab, np.float32)
        plugin.check(plugin.L.katali_cuda_download(lg.ctypes.data, ptr, lg.nbytes))
        assert rel_l2(lg, lc[i]) <= 1e-5, (i, rel_l2(lg, lc[i]))
        assert tok == int(ic[i]), i
    dm.close()
