"""Failure path of the decode loop on the device, without a GPU fault.

Every wait inside the decode loop kernel is bounded and reports through the
session's error word (src/engine.cc:231-239 is the reference's error
contract: no exception crosses the C ABI, failure is NULL / < 0 with the text
in last_error).  Here a test-only launch setting leaves one tagged word of the
first qkv phase unpublished (RPGB_TEST_DROP_WORD) and shortens the tagged-word
wait limit (RPGB_TEST_WAIT_LIMIT), so the attention phase's wait for that
word runs out: the kernel sets its error flag, every block leaves at its next
check, and the host raises.  The context stays usable; the session's length
is back at the prompt, and the next generate -- directly or through
rpg_engine_generate, which starts the session over after a failed decode as
the reference does after a failed prefill (src/engine.cc:531-537) -- gives
the same tokens as a fresh session.
"""

import ctypes
import json

import pytest

from rpgbarenginecuda_b200 import EngineError, Model, SampleOptions, Session, synthetic

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

GREEDY = SampleOptions(0.0, 0, 1.0)


def fault_on(monkeypatch):
    monkeypatch.setenv("RPGB_TEST_DROP_WORD", "1")
    monkeypatch.setenv("RPGB_TEST_WAIT_LIMIT", "65536")


def fault_off(monkeypatch):
    monkeypatch.delenv("RPGB_TEST_DROP_WORD", raising=False)
    monkeypatch.delenv("RPGB_TEST_WAIT_LIMIT", raising=False)


def test_wait_runs_out_and_session_recovers(tiny_model, monkeypatch):
    m = Model(tiny_model, 0, 512)
    s = Session(m, 512)
    toks = synthetic.seeded_tokens(21, 0, m.vocab)
    s.prefill(toks)
    fault_on(monkeypatch)
    with pytest.raises(EngineError, match="bounded device wait gave up"):
        s.generate(GREEDY, 0, 8)
    fault_off(monkeypatch)
    assert len(s) == 21  # nothing of the failed launch is kept
    with pytest.raises(EngineError, match="run a prefill first"):
        s.generate(GREEDY, 0, 8)  # its logits are gone too
    s.set_len(0)
    s.prefill(toks)
    ids = s.generate(GREEDY, 0, 8)
    fresh = Session(m, 512)
    fresh.prefill(toks)
    assert list(ids) == list(fresh.generate(GREEDY, 0, 8))
    # the next launch of the same session still runs many steps correctly
    more = s.generate(GREEDY, 0, 8)
    assert list(more) == list(fresh.generate(GREEDY, 0, 8))
    fresh.close()
    s.close()
    m.close()


def test_abi_generate_fails_cleanly_then_recovers(tiny_model, monkeypatch):
    from rpgbarenginecuda_b200._lib import load_engine

    L = load_engine()
    mh = L.rpg_engine_load_model(tiny_model.encode(), json.dumps({"context": 512, "device": 0}).encode())
    assert mh >= 0, L.rpg_engine_last_error()
    req = json.dumps({"messages": [{"role": "user", "content": "Hello there"}], "max_tokens": 8,
                      "temperature": 0.0}).encode()

    def generate(sh):
        p = L.rpg_engine_generate(sh, req)
        if not p:
            return None
        out = ctypes.string_at(p).decode()
        L.rpg_engine_free(p)
        return json.loads(out)

    sh = L.rpg_engine_session_create(mh, json.dumps({"max_seq": 512}).encode())
    assert sh >= 0
    fault_on(monkeypatch)
    assert generate(sh) is None
    assert b"bounded device wait gave up" in L.rpg_engine_last_error()
    fault_off(monkeypatch)
    got = generate(sh)
    sh2 = L.rpg_engine_session_create(mh, json.dumps({"max_seq": 512}).encode())
    want = generate(sh2)
    assert got is not None and got == want
    L.rpg_engine_session_destroy(sh)
    L.rpg_engine_session_destroy(sh2)
    L.rpg_engine_unload_model(mh)
