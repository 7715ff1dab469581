"""End-to-end text generation through Minima's own chat front end (chat.c,
unmodified; tests/chat_e2e_main.c builds the model and trains the
tokenizer): the build linked against the drop-in generate (the B200 token
loop) must print the same transcript as the build linked against the
reference generate.c, for the CHAT_* console protocol (chat.c:179-366:
history, /clear, Generation Lab /test settings, stop sequences, sampling
with penalties and n-gram bans, greedy) and for the generation diagnostics
(chat.c:457-556: next-token inspection, greedy repeatability, seeded
sampling).  Lines that carry wall-clock figures are left out of the
comparison.
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_BIN = os.path.join(ROOT, "oracle", "_ref", "chat_e2e_ref")
CUDA_BIN = os.path.join(ROOT, "oracle", "_ref", "chat_e2e_cuda")

SCRIPT = "\n".join([
    "hello there, how is the weather?",
    "what do cats like?",
    "/test 0.7 20 0.95 1.2 32",
    "the river",
    "/clear",
    "count to five",
    "/test 1.0 1 1.0 1.0 24",
    "Once upon a time",
    "thank you",
    "/quit",
]) + "\n"


def transcript(binary, mode, stdin=""):
    if not os.path.exists(binary):
        pytest.skip(f"{os.path.basename(binary)} not built (make -C oracle chat_e2e)")
    r = subprocess.run([binary, mode], input=stdin.encode(), capture_output=True, timeout=300)
    assert r.returncode == 0, r.stderr.decode(errors="replace")[-2000:]
    err = r.stderr.decode(errors="replace")
    assert "drop-in:" not in err, err[-2000:]
    keep = []
    for line in r.stdout.decode("latin-1").splitlines():
        if line.startswith("CHAT_STATS:") or "elapsed:" in line or line.startswith("BPE finished"):
            continue
        keep.append(line)
    return keep


def test_chat_console_reference_build():
    """The reference build speaks the protocol (CPU only)."""
    lines = transcript(REF_BIN, "console", SCRIPT)
    assert lines.count("CHAT_READY") >= 6
    assert sum(l.startswith("BOT: ") for l in lines) == 4
    assert sum(l.startswith("TEST: ") for l in lines) == 2
    assert lines[-1] == "CHAT_CLOSED"


@pytest.mark.gpu
def test_chat_console_matches_reference(gpu):
    """Greedy replies (repetition penalty, n-gram bans, stop sequence, the
    /test lab settings of the script, multi-turn history): identical."""
    assert transcript(CUDA_BIN, "console", SCRIPT) == transcript(REF_BIN, "console", SCRIPT)


@pytest.mark.gpu
def test_chat_sampled_console_protocol(gpu):
    """Seeded top-k/top-p sampling: the same protocol lines, and at least 5 of
    the 6 replies identical.  A sampled reply is identical while every draw
    falls on the same side of the same cumulative-probability boundaries,
    which fp32 logits computed in another order do not guarantee on a
    random-init model's near-uniform distributions (measured: 6 of 6)."""
    got = transcript(CUDA_BIN, "sampled", SCRIPT)
    want = transcript(REF_BIN, "sampled", SCRIPT)
    kinds = lambda ls: [l.split(":")[0] if l[:4] in ("BOT:", "TEST") else l for l in ls
                        if l.startswith(("CHAT_", "BOT:", "TEST"))]
    assert kinds(got) == kinds(want)
    replies = lambda ls: [l for l in ls if l.startswith(("BOT:", "TEST:"))]
    same = sum(a == b for a, b in zip(replies(got), replies(want)))
    print(f"sampled replies identical: {same}/{len(replies(want))}")
    assert same >= len(replies(want)) - 1


@pytest.mark.gpu
def test_chat_generation_diagnostics_match_reference(gpu):
    """Next-token inspection (top-10 ids), greedy continuations and the
    greedy repeatability check: identical."""
    got = transcript(CUDA_BIN, "bench")
    want = transcript(REF_BIN, "bench")
    assert "Deterministic greedy check: PASS (all prompts reproduced exactly)" in want
    pick = lambda ls: [l for l in ls if "greedy" in l or "Prompt:" in l or " id=" in l]
    assert pick(got) == pick(want)
    assert got[-1] == want[-1]
