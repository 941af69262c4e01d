"""Weight loader (InferenceEngine.load / xl_engine_load): the raw-fp32 tree of
the reference's exporter, read by worker threads into pinned buffers and copied
on their own streams.  Any number of workers must give the same device
weights; a missing or short file fails the load with the file's name
(RuntimeError: the reference's Tensor::load throws std::runtime_error there,
src/tensor.cu:116,121)."""
import os
import shutil

import numpy as np
import pytest

import xl_synth as S

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng_mod(built):
    import llm_cpp_engine

    return llm_cpp_engine


@pytest.mark.parametrize("shape_name", ["TINY", "WIDE2"])
def test_load_threads_give_identical_weights(eng_mod, shape_name):
    sh = getattr(S, shape_name)
    wdir = S.write_weight_tree(f"/tmp/xl_weights/{shape_name.lower()}", sh)
    ids = S.prompt_ids(3, 21, sh.vocab)
    out = []
    for threads in (1, 3, 4, 16):
        eng = eng_mod.InferenceEngine("cuda", **sh.engine_kwargs())
        eng.set_option("load_threads", threads)
        eng.load(wdir)
        assert eng.last_load_s() > 0.0
        tok = eng.next_token(ids, top_p=0.0, repetition_penalty=1.0)
        kb, vb = eng.kv(1, eng.ctx_len(), sh.heads)
        out.append((tok, np.frombuffer(eng.last_logits(), np.float32).copy(), bytes(kb), bytes(vb)))
    for o in out[1:]:
        assert o[0] == out[0][0]
        assert np.array_equal(o[1], out[0][1])
        assert o[2] == out[0][2] and o[3] == out[0][3]


def test_load_reports_missing_and_short_files(eng_mod, tmp_path):
    sh = S.TINY
    src = S.write_weight_tree("/tmp/xl_weights/tiny", sh)
    bad = tmp_path / "tree"
    shutil.copytree(src, bad)
    victim = bad / "blocks" / "1" / "ffn" / "W2" / "weight.bin"
    with open(victim, "r+b") as f:
        f.truncate(os.path.getsize(victim) - 4)
    eng = eng_mod.InferenceEngine("cuda", **sh.engine_kwargs())
    with pytest.raises(RuntimeError, match="blocks/1/ffn/W2/weight.bin"):
        eng.load(str(bad))
    os.remove(victim)
    with pytest.raises(RuntimeError, match="blocks/1/ffn/W2/weight.bin"):
        eng.load(str(bad))
    eng.load(src)  # the engine stays usable
    assert eng.next_token(S.prompt_ids(1, 5, sh.vocab), top_p=0.0) >= 0
