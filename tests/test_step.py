"""vp_step (one decode step from host memory: state and tree in, pass, state and this pass's
committed tokens out) gives the same state and committed tokens as the separate calls it stands
for: vp_write_state, vp_pass, vp_read_state, vp_read_tokens."""
import numpy as np
import pytest

from instantllm_b200 import synth
from instantllm_b200._lib import STATE_FIELDS, VpState

pytestmark = pytest.mark.gpu


def test_step_matches_separate_calls():
    from instantllm_b200.engine import VerifyEngine

    V = 4096
    eng = VerifyEngine(synth.make_weights("q4", n_layers=2, vocab=V, seed=51), max_ctx=256, max_steps=64)
    eng.begin(0, 32)
    eng.prefill((synth.make_prompt(40, seed=51) % V).tolist())
    first = eng.tokens(1)[0]
    snap = eng.snapshot()
    rng = np.random.default_rng(51)
    trees = [synth.tree_to_buffer(synth.seeded_tree(rng, [first] * 9, n=16, vocab=V)) for _ in range(3)]

    want = []
    eng.restore(snap, on_device=False)
    for t in trees:
        eng.pass_(t)
        st = eng.state()
        want.append((st, eng.tokens(st["step"])))

    got = []
    st = eng.step(trees[0], snap[0])  # from the snapshot, then continuing from the device state
    got.append((st.as_dict(), eng.tokens(st.step)))
    returned = list(eng.tokens(1)) + eng.last_tokens()  # the prefill's token, then each pass's
    for t in trees[1:]:
        st = eng.step(t)
        got.append((st.as_dict(), eng.tokens(st.step)))
        returned += eng.last_tokens()
    assert got == want
    assert returned == want[-1][1]  # the tokens vp_step handed back are the committed stream

    # a request that has stopped commits nothing: vp_step hands back no tokens
    done = dict(want[-1][0], done=1)
    st = eng.step(trees[0], VpState(*[done[n] for n in STATE_FIELDS]))
    assert st.step == done["step"] and eng.last_tokens() == []
    eng.close()
