"""The drop-in boundary exercised by the reference's own caller: the
reference CLI (cli/main.c) linked against hako_b200/host/hakm_model_cuda.c in
place of src/model.c, run as a greedy raw completion (`-t 0 --raw`:
src/sample.c's argmax over the logits hakm_forward returns).

The drop-in's forward pass is bit-identical to the reference's, so the ids it
is fed (prompt, then its own picks, logged) equal the reference's greedy
continuation of the same prompt ids, and the two CLIs print the same bytes."""
import os
import subprocess

import pytest

from oracle.oracle import DROPIN_CLI, REF_CLI

pytestmark = pytest.mark.gpu


def _run(cli, path, n, prompt, env_extra=None):
    env = dict(os.environ, HAKM_THREADS=str(min(os.cpu_count() or 1, 16)))
    env.update(env_extra or {})
    r = subprocess.run([cli, path, "-t", "0", "--raw", "--ctx", "256", "-n", str(n), prompt],
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
