"""Chat driver on the B200 (synthetic weights, the seeded synthetic tokenizer
of tests/golden/make_tokenizer_golden.py): its token stream — prefill, host
sample of the first token with the RNG advanced over the prompt, device decode
steps — equals main.cu's loop emulated one position at a time (forward, then
sample() after every position, prompt positions included), greedy and
sampled; the printed text is the pieces of the generated tokens."""
import importlib.util
import io
import os
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_tokenizer_golden as G  # noqa: E402


def _mod(name, file):
    spec = importlib.util.spec_from_file_location(name, os.path.join(REPO, "qwen600-rocm-inference_b200", file))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _reference_loop(qb, eng, ids, sp, seed, n_new):
    """main.cu:141-146 one position at a time: forward(token, pos), next =
    sample(logits) after every position; returns the first n_new tokens after
    the prompt."""
    rng, nxt, gen = seed, None, []
    pos = 0
    while len(gen) < n_new:
        token = ids[pos] if pos < len(ids) else nxt
        if pos >= len(ids):
            gen.append(token)
        lg = eng.forward(token, pos)
        nxt, rng = qb.sample_host(lg, sp, rng)
        pos += 1
    return gen


@pytest.mark.parametrize("temperature,top_p,top_k,seed", [(0.0, 0.95, 20, 7), (0.6, 0.95, 20, 1234), (1.0, 0.9, 40, 99)])
def test_chat_turn_matches_reference_loop(qb, checkpoint, tmp_path, temperature, top_p, top_k, seed):
    T = _mod("qwen_tokenizer", "tokenizer.py")
    C = _mod("qwen_chat", "chat.py")
    G.write_model_dir(str(tmp_path))
    tok = T.Tokenizer(str(tmp_path / "tokenizer.bin"))
    templates = T.load_templates(str(tmp_path), False)
    sp = qb.Sampling(temperature, top_p, top_k)
    out = io.StringIO()
    n_new = 24
    a = qb.Engine(checkpoint, 0)
    b = qb.Engine(checkpoint, 0)
    try:
        chat = C.Chat(a, tok, templates, sp, seed, out=out, color=False)
        gen, text, tps = chat.turn("kato rise <think>anon</think>", "be brief", max_new=n_new)
        ids = tok.encode(T.render(templates[1], "be brief", "kato rise <think>anon</think>"))
        assert len(ids) < 65      # the prompt goes through per-position decode launches: same logits as forward()
        ref = _reference_loop(qb, b, ids, sp, seed, len(gen))
        assert gen == ref
        assert 1 <= len(gen) <= n_new   # an EOS may end the turn early
        assert text == b"".join(tok.decode(t) for t in gen)
        assert "tk/s" in out.getvalue() and tps > 0
        # a second turn starts a new sequence at position 0 with the user template
        gen2, _, _ = chat.turn("again", max_new=8)
        assert len(gen2) >= 1
    finally:
        a.close(); b.close(); tok.close()
