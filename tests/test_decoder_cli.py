"""The loom_private decoder drop-in executable (cuda-elastic_b200/decoder_b200)
on the reference's own test list (applications/loom_private/decoder/tests/
run_tests.sh): correct runs at wrapping and ragged shapes in Direct and Graph
mode, invalid dimensions and usage (exit 2, before any device work, so those
run on the CPU), injected faults reported with indices and expected/actual
values (exit 1), the large check with the reference's digest, and the
RESULT record of check, bench and profile (lp_harness.cuh:426-596)."""
import json
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "cuda-elastic_b200", "decoder_b200")


def run(*args, timeout=900):
    r = subprocess.run([EXE] + list(args), capture_output=True, text=True, timeout=timeout)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT ")]
    record = json.loads(lines[-1][len("RESULT "):]) if lines else None
    return r, record


def sets(**kw):
    out = []
    for k, v in kw.items():
        out += ["--set", f"{k}={v}"]
    return out


# ---------------------------------------------------------------- CPU: usage

@pytest.mark.parametrize("args,pattern", [
    (sets(vocab=1, width=8), "vocab must satisfy"),
    (sets(vocab=17, width=16), "vocab must satisfy"),
    (sets(steps=1, width=32, vocab=8), "steps must be"),
    (sets(batch=0), "batch must be"),
    (sets(width=0), "width must be"),
    (sets(batch=1, width=16777201, vocab=2, steps=2), "width must be"),
    (sets(batch=1048576), "GiB"),
    (sets(batch="abc"), "not an integer"),
    (sets(rows=4), "unsupported --set key 'rows'"),
    (["--preset", "smoke"] + sets(width=32, vocab=8), "unknown preset 'smoke'"),
    (sets(fault=4), "fault must be 0, 1, 2 or 3"),
    (["--action", "bench"], "needs --launch direct or --launch graph"),
    (["--action", "profile", "--launch", "both"], "needs --launch direct or --launch graph"),
    (["--action", "bench", "--launch", "graph"] + sets(batch=3), "--set is only valid with --action check"),
    (["--launch", "sideways"], "--launch must be"),
    (["--iterations", "0"], "--iterations expects an integer >= 1"),
    (["--asset", "model=x"], "unsupported --asset name 'model'"),
    (["--set", "novalue"], "expects key=value"),
    (["--json-out"], "needs a value"),
    (["--frobnicate", "1"], "unknown option --frobnicate"),
])
def test_usage_errors_exit_2(args, pattern):
    r, rec = run(*args, timeout=60)
    assert r.returncode == 2, (r.returncode, r.stderr)
    assert pattern in r.stderr, r.stderr
    assert rec is None


def test_help_exits_0():
    r, _ = run("--help", timeout=60)
    assert r.returncode == 0 and "--action check|bench|profile" in r.stdout


# ---------------------------------------------------------------- GPU: runs

@pytest.mark.gpu
@pytest.mark.parametrize("name,args,pattern", [
    ("wraparound", sets(batch=40, width=96, vocab=16, steps=5), "PASS: 0/200 tokens wrong"),
    ("minimum", sets(batch=3, width=2, vocab=2, steps=2), "PASS"),
    ("square", sets(batch=1030, width=1000, vocab=1000, steps=3), "PASS"),
    ("wide", sets(batch=1, width=4100, vocab=300, steps=2), "PASS"),
    ("graph-only", ["--launch", "graph"] + sets(batch=70, width=200, vocab=33, steps=4),
     "graph invocation 2: PASS"),
])
def test_correct_runs(name, args, pattern):
    r, rec = run(*args)
    assert r.returncode == 0, r.stderr
    assert pattern in r.stderr, r.stderr
    assert rec["status"] == "pass" and rec["outputs_agree"] is True
    assert rec["schema"] == "loom_private.result/1"
    assert rec["identity"] == "loom-private/llama2c-decoder"
    modes = {c["launch"] for c in rec["checks"]}
    assert modes == ({"graph"} if name == "graph-only" else {"direct", "graph"})
    assert len({c["digest"] for c in rec["checks"]}) == 1
    assert rec["overrides"] == {k.split("=")[0]: int(k.split("=")[1])
                                for k in args[1::2] if "=" in k}


@pytest.mark.gpu
@pytest.mark.parametrize("fault,pattern", [
    (1, "token mismatch sequence 39 step 4: expected 12, actual 13"),
    (2, "invariant failure sequence 20 step 4"),
    (3, "probability mismatch sequence 0 step 4 index 8: expected"),
])
def test_injected_faults_are_reported(fault, pattern):
    r, rec = run(*sets(batch=40, width=96, vocab=16, steps=5, fault=fault))
    assert r.returncode == 1, r.stderr
    assert pattern in r.stderr, r.stderr
    assert rec["status"] == "fail"


@pytest.mark.gpu
def test_large_check_matches_reference_digest(tmp_path):
    """The large preset in both launch modes: every check passes and every
    digest equals the reference's recorded large-shape digest
    (decoder/README.md:183-185)."""
    out = tmp_path / "check.json"
    r, rec = run("--json-out", str(out))
    assert r.returncode == 0, r.stderr
    assert rec["status"] == "pass"
    assert rec["dimensions"]["classifier_macs_per_step"] == 137438953472
    assert rec["dimensions"]["model_bytes"] == 1073807360
    assert {c["digest"] for c in rec["checks"]} == {"4fcc3e102976547b"}
    assert json.loads(out.read_text()) == rec


@pytest.mark.gpu
@pytest.mark.parametrize("launch", ["direct", "graph"])
def test_bench_and_profile_records(launch):
    r, rec = run("--action", "bench", "--launch", launch, "--iterations", "2", "--warmup", "1",
                 *([]))
    assert r.returncode == 0, r.stderr
    assert rec["status"] == "unvalidated_bench" and rec["iterations"] == 2
    for scope in ("application", "compute"):
        t = rec["timing"][scope]
        assert len(t["single_us"]) == 2 and t["batch_per_iteration_us"] > 0
    # the application scope downloaded the generated tokens of the last run
    assert rec["output_digest"] != f"{0:016x}"
    r, rec = run("--action", "profile", "--launch", launch)
    assert r.returncode == 0, r.stderr
    assert rec["status"] == "profile" and rec["timing"] is None
