"""CLI commands (CPU): synth/inspect/adjudicate and guard wrapping a child process."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run(*args, **kw):
    env = dict(os.environ, PYTHONPATH=ROOT)
    return subprocess.run([sys.executable, "-m", "fak_b200", *args], cwd=ROOT, env=env, capture_output=True,
                          text=True, timeout=300, **kw)


def test_synth_inspect_adjudicate(tmp_path):
    out = str(tmp_path / "m.gguf")
    assert run("synth", "tiny-llama", out, "--mix", "q8_0").returncode == 0
    r = run("inspect", out)
    info = json.loads(r.stdout)
    assert info["config"]["n_layers"] == 2 and "Q8_0" in info["bytes_by_type"]
    r = run("adjudicate", '{"tool": "Bash", "args": {"command": "sudo reboot"}}')
    assert r.returncode == 3 and json.loads(r.stdout)["reason"] == "POLICY_BLOCK"
    assert run("adjudicate", '{"tool": "Read", "args": {"path": "x"}}').returncode == 0


def test_guard_wraps_agent_with_cpu_model(tmp_path):
    out = str(tmp_path / "m.gguf")
    assert run("synth", "tiny-qwen2", out, "--mix", "f32").returncode == 0
    agent = ("import os, json, urllib.request as u;"
             "b=os.environ['OPENAI_BASE_URL'];"
             "req=u.Request(b+'/chat/completions', data=json.dumps({'messages':[{'role':'user','content':'hi'}],"
             "'max_tokens':3}).encode(), headers={'content-type':'application/json'});"
             "print(json.load(u.urlopen(req))['object']);"
             "req=u.Request(os.environ['FAK_GATEWAY_URL']+'/v1/fak/adjudicate', data=json.dumps({'tool':'rm_all',"
             "'args':{}}).encode(), headers={'content-type':'application/json'});"
             "print(json.load(u.urlopen(req))['reason'])")
    journal = str(tmp_path / "j.jsonl")
    r = run("guard", "--gguf", out, "--cpu", "--journal", journal, "--", sys.executable, "-c", agent)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "chat.completion" in r.stdout and "DEFAULT_DENY" in r.stdout
    summary = json.loads(r.stderr.strip().splitlines()[-1])
    assert summary["denied"] == 1 and summary["journal_chain_ok"]
