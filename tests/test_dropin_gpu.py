"""The drop-in boundary exercised by the reference's own caller: the
reference CLI (cli/main.c) linked against hako_b200/host/hakm_model_cuda.c in
place of src/model.c (and src/sample.c's sample_token renamed, so the pick is
made on the device) and hakm_tok_dropin.c (libhakm_tok, the Qwen2 tokenizer)
in place of src/bpe.c, run as a raw completion.

The drop-in defers the fed ids until sample_token needs their logits (the
prompt then runs as one batched pass), and its forward pass and sampler are
bit-identical to the reference's: the ids it is fed (prompt, then its own
picks, logged) equal the reference's greedy continuation of the same prompt
ids, and the two CLIs print the same bytes, greedy (`-t 0`), with
temperature / top-k / top-p sampling from a fixed seed, and with the
deferred feed switched off (HAKMC_EAGER=1)."""
import os
import subprocess

import pytest

from oracle.oracle import DROPIN_CLI, REF_CLI

pytestmark = pytest.mark.gpu


def _run(cli, path, n, prompt, env_extra=None, sampling=("-t", "0")):
    env = dict(os.environ, HAKM_THREADS=str(min(os.cpu_count() or 1, 16)))
    env.update(env_extra or {})
    r = subprocess.run([cli, path, *sampling, "--raw", "--ctx", "256", "-n", str(n), prompt],
                       capture_output=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr.decode(errors="replace")[-400:]
    return r.stdout


@pytest.mark.parametrize("preset,n", [("small", 40), ("3b", 24)])
def test_reference_cli_over_dropin(cuda, tmp_path, preset, n):
    from hako_b200 import synth
    if not (os.path.exists(REF_CLI) and os.path.exists(DROPIN_CLI)):
        pytest.skip("oracle/_ref CLIs not built (make -C oracle ref dropin)")
    path = synth.cached_model(synth.PRESETS[preset])
    prompt = "the quick brown fox jumps over"
    log = tmp_path / "ids.txt"
    # -n 0: the log holds exactly the prompt's ids (cli/main.c feed())
    _run(DROPIN_CLI, path, 0, prompt, {"HAKMC_TOKEN_LOG": str(log)})
    prompt_ids = [int(x) for x in log.read_text().split()]
    assert prompt_ids
    ours = _run(DROPIN_CLI, path, n, prompt, {"HAKMC_TOKEN_LOG": str(log)})
    ids = [int(x) for x in log.read_text().split()]
    assert ours.startswith(prompt.encode()) and len(ours) > len(prompt)
    assert ids[:len(prompt_ids)] == prompt_ids
    fed = ids[len(prompt_ids):]  # generate(): each pick is fed back (until eos)
    assert fed
    ref_stream, _ = ref_greedy(path, prompt_ids, n)
    assert fed == ref_stream[:len(fed)]
    assert ours == _run(REF_CLI, path, n, prompt)


@pytest.mark.parametrize("sampling", [("-t", "0.8", "-k", "40", "-p", "0.9", "-s", "1234"),
                                      ("-t", "1.1", "-k", "0", "-p", "0.95", "-s", "77"),
                                      ("-t", "0.6", "-k", "5", "-p", "0", "-s", "9")])
def test_reference_cli_sampling_over_dropin(cuda, sampling):
    """Temperature / top-k / top-p sampling from a fixed seed: the drop-in's
    device sampler draws the reference's ids, so both CLIs print the same
    bytes (and the generator state advances alike, step after step)."""
    from hako_b200 import synth
    if not (os.path.exists(REF_CLI) and os.path.exists(DROPIN_CLI)):
        pytest.skip("oracle/_ref CLIs not built (make -C oracle ref dropin)")
    path = synth.cached_model(synth.PRESETS["small"])
    prompt = "once upon a time there was a"
    ours = _run(DROPIN_CLI, path, 48, prompt, sampling=sampling)
    assert ours == _run(REF_CLI, path, 48, prompt, sampling=sampling)


def test_reference_cli_over_dropin_qwen2_tokenizer(cuda, tmp_path):
    """The prompt reaches the model as the Qwen2 tokenizer's ids
    (hako_b200.tokenizer over the model file's tokenizer blob): digit,
    punctuation and whitespace runs and contractions included; the
    continuation of those ids is the reference model's."""
    from hako_b200 import synth
    from hako_b200.tokenizer import Tokenizer
    if not os.path.exists(DROPIN_CLI):
        pytest.skip("oracle/_ref/hakm_cuda not built (make -C oracle dropin)")
    path = synth.cached_model(synth.PRESETS["small"])
    prompt = "It's 2024!!!  Numbers: 12345,\n\nand don't   stop... the end"
    want = Tokenizer.from_mlf2(path).encode(prompt)
    log = tmp_path / "ids.txt"
    _run(DROPIN_CLI, path, 0, prompt, {"HAKMC_TOKEN_LOG": str(log)})
    assert [int(x) for x in log.read_text().split()] == want
    out = _run(DROPIN_CLI, path, 24, prompt, {"HAKMC_TOKEN_LOG": str(log)})
    assert out.startswith(prompt.encode())
    ids = [int(x) for x in log.read_text().split()]
    assert ids[:len(want)] == want
    fed = ids[len(want):]
    assert fed
    ref_stream, _ = ref_greedy(path, want, 24)
    assert fed == ref_stream[:len(fed)]


def test_reference_cli_over_dropin_eager(cuda):
    """HAKMC_EAGER=1: every hakm_forward runs at once and copies its logits
    (the reference's contract for c->logits); same bytes."""
    from hako_b200 import synth
    if not (os.path.exists(REF_CLI) and os.path.exists(DROPIN_CLI)):
        pytest.skip("oracle/_ref CLIs not built (make -C oracle ref dropin)")
    path = synth.cached_model(synth.PRESETS["small"])
    prompt = "the quick brown fox jumps over"
    assert _run(DROPIN_CLI, path, 32, prompt, {"HAKMC_EAGER": "1"}) == _run(REF_CLI, path, 32, prompt)


def ref_greedy(path, prompt_ids, n):
    """The reference's greedy picks after the prompt and each pick's top-2 margin."""
    import numpy as np
    from oracle.oracle import RefModel
    ref = RefModel(path, 256)
    logits, am = None, None
    for t in prompt_ids:
        logits, am = ref.forward(t)
    stream, gaps = [], []
    for _ in range(n):
        srt = np.sort(logits)
        stream.append(am)
        gaps.append(float(srt[-1] - srt[-2]))
        logits, am = ref.forward(am)
    ref.close()
    return stream, gaps


def test_dropin_info_and_bad_path(cuda):
    from hako_b200 import synth
    if not os.path.exists(DROPIN_CLI):
        pytest.skip("oracle/_ref/hakm_cuda not built")
    path = synth.cached_model(synth.PRESETS["tiny"])
    r = subprocess.run([DROPIN_CLI, path, "--info"], capture_output=True, timeout=120)
    assert r.returncode == 0 and b"layers" in r.stderr
    r = subprocess.run([DROPIN_CLI, "/nonexistent.mlf2", "--info"], capture_output=True, timeout=120)
    assert r.returncode != 0
