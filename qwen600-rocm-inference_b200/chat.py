"""Chat driver: text in, text out, on the B200 engine — the reference's chat
loop (main.cu:85-205) and command line (main.cu:236-282).

    python qwen600-rocm-inference_b200/chat.py <model_dir> [-t 0.6] [-p 0.95] [-k 20] [-s seed]
                                               [-i prompt] [-y system_prompt] [-r 0|1]
                                               [--checkpoint PATH] [--device D] [--max-new N] [--no-color]

<model_dir> holds tokenizer.bin and the template_*.txt files (and
model.safetensors, unless --checkpoint names another file).  Each user turn
starts a new sequence at position 0, as in the reference: the prompt is
rendered with the user (or, on the first turn with -y, the system) template,
encoded, prefilled, then tokens are sampled until EOS.  The stream of tokens
equals the reference's for the same seed: the reference samples after every
prompt position too (one xorshift64* draw each when sampling is random), so
the RNG is advanced by one draw per prompt position before the first
generated token.  --max-new (default: until the context is full) bounds a
turn; the reference has no such bound and in -i mode restarts the prompt when
the context fills.
"""
import argparse
import os
import sys
import time

import importlib.util

HERE = os.path.dirname(os.path.abspath(__file__))


def _load(name, file):
    spec = importlib.util.spec_from_file_location(name, os.path.join(HERE, file))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


YELLOW, BOLD_RED, GREEN, RESET = "\033[33m", "\033[1;31m", "\033[32m", "\033[0m"
MASK64 = (1 << 64) - 1


def rng_advance(state, k):
    """k state updates of the sampler's xorshift64* generator (sampler.h
    random_u32: the shifts 12, 25, 27 on a 64-bit state)."""
    for _ in range(k):
        state ^= state >> 12
        state ^= (state << 25) & MASK64
        state ^= state >> 27
    return state & MASK64


def parse_args(argv):
    """main.cu:243-270: positional model_dir, then -x value pairs; seed <= 0 ->
    the current time; temperature < 0 -> 0; top_p outside [0, 1] -> 0.95."""
    ap = argparse.ArgumentParser(prog="chat.py", description=__doc__.split("\n\n")[0])
    ap.add_argument("model_dir")
    ap.add_argument("-t", type=float, default=0.6, dest="temperature")
    ap.add_argument("-p", type=float, default=0.95, dest="top_p")
    ap.add_argument("-k", type=int, default=20, dest="top_k")
    ap.add_argument("-s", type=int, default=0, dest="seed")
    ap.add_argument("-i", default=None, dest="prompt")
    ap.add_argument("-y", default=None, dest="system_prompt")
    ap.add_argument("-r", type=int, default=0, dest="thinking")
    ap.add_argument("--checkpoint", default=None)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--max-new", type=int, default=None)
    ap.add_argument("--no-color", action="store_true")
    a = ap.parse_args(argv)
    if a.seed <= 0:
        a.seed = int(time.time()) & 0xFFFFFFFF
    if a.temperature < 0:
        a.temperature = 0.0
    if a.top_p < 0 or a.top_p > 1.0:
        a.top_p = 0.95
    return a


class Chat:
    """One chat session: engine + tokenizer + templates + sampler state."""

    def __init__(self, engine, tokenizer, templates, sampling, seed, thinking=False, out=None, color=True):
        self.qb = _load("qwen_b200", "qwen_b200.py")
        self.T = _load("qwen_tokenizer", "tokenizer.py")
        self.eng, self.tok = engine, tokenizer
        self.user_t, self.system_t = templates
        self.sp, self.rng = sampling, seed & MASK64
        self.thinking, self.out, self.color = bool(thinking), out, color
        self.first_turn = True

    def _emit(self, s):
        if self.out is not None:
            self.out.write(s)
            self.out.flush()

    def _c(self, code):
        return code if self.color else ""

    def turn(self, user_prompt, system_prompt=None, max_new=None):
        """One user turn (main.cu:118-200).  Returns (generated token ids, the
        bytes printed for them, tokens per second as the reference reports it)."""
        if self.first_turn and system_prompt:
            text = self.T.render(self.system_t, system_prompt, user_prompt)
        else:
            text = self.T.render(self.user_t, user_prompt)
        self.first_turn = False
        ids = self.tok.encode(text)
        if not ids:
            raise ValueError("the rendered prompt encodes to no tokens")
        n = len(ids)
        seq_len = self.qb.SEQ_LEN
        if n >= seq_len:
            raise ValueError(f"prompt of {n} tokens does not fit the {seq_len}-position context")
        limit = seq_len - n if max_new is None else min(max_new, seq_len - n)
        random = not (self.sp.temperature == 0.0 or self.sp.top_k == 1)
        logits = self.eng.prefill(ids, 0, want_logits=True)
        if random:
            self.rng = rng_advance(self.rng, n - 1)   # the reference samples after each of the first n - 1 positions
        nxt, self.rng = self.qb.sample_host(logits, self.sp, self.rng)
        t0 = time.perf_counter()
        gen, text_out = [], []
        in_think, in_bold = self.thinking, False
        if in_think:
            self._emit(self._c(YELLOW))
        pos = n
        while len(gen) < limit:
            token = nxt
            gen.append(token)
            piece = self.tok.decode(token)
            text_out.append(piece)
            if piece == b"</think>":
                in_think = False
                if not in_bold:
                    self._emit(self._c(RESET))
            else:
                parts = piece.split(b"**")
                for j, part in enumerate(parts):
                    self._emit(part.decode("utf-8", errors="replace"))
                    if j + 1 < len(parts):
                        in_bold = not in_bold
                        self._emit(self._c(BOLD_RED) if in_bold else (self._c(YELLOW) if in_think else self._c(RESET)))
            if len(gen) >= limit or pos >= seq_len:
                break
            nxt, self.rng = self.eng.decode_step(token, pos, self.sp, self.rng)
            pos += 1
            if nxt == self.tok.eos_token_id:
                break
        dt = time.perf_counter() - t0
        tps = (len(gen) - 1) / dt if len(gen) > 1 and dt > 0 else 0.0
        self._emit(f"\n\n{self._c(GREEN)}[{tps:.2f} tk/s, {len(gen) - 1} tokens in {dt:.2f}s]{self._c(RESET)}\n")
        return gen, b"".join(text_out), tps


def main(argv=None):
    a = parse_args(sys.argv[1:] if argv is None else argv)
    qb = _load("qwen_b200", "qwen_b200.py")
    T = _load("qwen_tokenizer", "tokenizer.py")
    ck = a.checkpoint or os.path.join(a.model_dir, "model.safetensors")
    tok = T.Tokenizer(os.path.join(a.model_dir, "tokenizer.bin"))
    templates = T.load_templates(a.model_dir, a.thinking)
    sp = qb.Sampling(a.temperature, a.top_p, a.top_k)
    with qb.Engine(ck, a.device) as eng:
        chat = Chat(eng, tok, templates, sp, a.seed, a.thinking, out=sys.stdout, color=not a.no_color)
        while True:
            if a.prompt is not None:
                user = a.prompt
            else:
                try:
                    user = input("\n>> ")
                except EOFError:
                    break
                if not user:
                    break
            sys.stdout.write("\n")
            chat.turn(user, a.system_prompt, a.max_new)
            sys.stdout.write("\n===================================\n")
            if a.prompt is not None:
                break
    tok.close()


if __name__ == "__main__":
    main()
