"""CLI flags: environment fallbacks (command line > CASCADIA_* env >
built-in default) and rejection of flag combinations that cannot run."""
import argparse

import pytest

from cascadia_b200 import cli


def _args(**kw):
    base = dict(model="tiny-llama", engine="llama", max_model_len=512, max_running=8,
                kv_blocks=0, kv_prefix_cache_size=0, kv_fraction=0.5, tp=1, pp=1, ep=1, spec=None,
                draft_model=None, prompt=None, prompt_ids=None)
    base.update(kw)
    return argparse.Namespace(**base)


def test_env_fallback_and_precedence(monkeypatch):
    monkeypatch.setenv("CASCADIA_MAX_RUNNING", "12")
    assert cli._env("MAX_RUNNING", 64, int) == 12
    monkeypatch.delenv("CASCADIA_MAX_RUNNING")
    assert cli._env("MAX_RUNNING", 64, int) == 64
    monkeypatch.setenv("CASCADIA_KV_FRACTION", "abc")
    with pytest.raises(SystemExit):
        cli._env("KV_FRACTION", 0.5, float)
    monkeypatch.delenv("CASCADIA_KV_FRACTION")
    # Defaults are read when the parser is built; the command line wins.
    monkeypatch.setenv("CASCADIA_MAX_MODEL_LEN", "777")
    p = argparse.ArgumentParser()
    cli._common(p)
    assert p.parse_args([]).max_model_len == 777
    assert p.parse_args(["--max-model-len", "99"]).max_model_len == 99


@pytest.mark.parametrize("kw, msg", [
    (dict(max_model_len=0), "positive"),
    (dict(kv_fraction=1.5), "kv-fraction"),
    (dict(kv_blocks=16, kv_prefix_cache_size=16), "prefix-cache"),
    (dict(engine="dsv4", tp=2), "one device"),
    (dict(spec="ngram", pp=2), "single stage"),
    (dict(spec="draft"), "draft-model"),
    (dict(model="llama-3.1-8b", tp=3), "must divide"),
    (dict(prompt_ids="1,2"), "needs --prompt"),
    (dict(ep=2), "sparse-MoE"),
    (dict(model="tiny-moe", ep=3), "must divide"),
    (dict(model="tiny-moe", ep=2, tp=2), "no --tp"),
])
def test_bad_combinations_rejected(kw, msg):
    with pytest.raises(SystemExit) as e:
        cli.validate_run_flags(_args(**kw))
    assert msg in str(e.value)


def test_good_combinations_pass():
    cli.validate_run_flags(_args())
    cli.validate_run_flags(_args(model="llama-3.1-8b", tp=8))
    cli.validate_run_flags(_args(tp=2, pp=2))
    cli.validate_run_flags(_args(spec="draft", draft_model="tiny-llama"))
