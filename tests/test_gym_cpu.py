"""Research gym: packages, budget, leases, research data parallelism, HTTP API and MCP (CPU)."""
import copy
import io
import json
import socket
import subprocess
import sys
import threading
import time
import zipfile
import base64

import pytest
import torch

from nexttransformer_b200.gym import contract
from nexttransformer_b200.gym.contract import GymError
from nexttransformer_b200.gym.package import candidate_from_package, make_package

PLUGIN = '''
import torch.nn.functional as F
from torch import nn
from nexttransformer_b200.models.shell import Linear


class SiluMLP(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.c_fc = Linear(config.width, config.mlp_width, bias=False)
        self.c_proj = Linear(config.mlp_width, config.width, bias=False)

    def forward(self, x):
        return self.c_proj(F.silu(self.c_fc(x)))


def ffn(config, layer):
    return SiluMLP(config)
'''


def _files(name="silu_probe", **extra):
    files = {"proposal.json": json.dumps({"name": "SiLU MLP", "summary": "probe"}),
             f"plugin/{name}/method.json": json.dumps({"name": name, "family": "others", "title": "SiLU probe"}),
             f"plugin/{name}/__init__.py": PLUGIN}
    files.update(extra)
    return files


def test_package_accepts_and_is_content_addressed():
    cid, method, proposal, files = candidate_from_package(make_package(_files()))
    cid2, *_ = candidate_from_package(make_package(_files()))
    assert cid == cid2 and method == "silu_probe" and proposal["name"] == "SiLU MLP"
    cid3, *_ = candidate_from_package(make_package(_files(**{"plugin/silu_probe/extra.py": "X = 1\n"})))
    assert cid3 != cid


def _zip_raw(entries):
    buf = io.BytesIO()
    with zipfile.ZipFile(buf, "w") as zf:
        for info, data in entries:
            zf.writestr(info, data)
    return base64.b64encode(buf.getvalue()).decode()


@pytest.mark.parametrize("bad", [
    lambda: make_package(_files(**{"../evil.py": "x"})),
    lambda: make_package(_files(**{"plugin/silu_probe/run.sh": "rm -rf /"})),
    lambda: make_package(_files(**{"plugin/silu_probe/w.py": b"\xff\xfe\x00binary"})),
    lambda: make_package(_files(**{"plugin/silu_probe/bad.py": "def f(:\n"})),
    lambda: make_package({k: v for k, v in _files().items() if k != "proposal.json"}),
    lambda: make_package(_files(**{"plugin/other/method.json": "{}"})),
    lambda: make_package({**_files(), "plugin/silu_probe/method.json": json.dumps({"name": "x", "family": "others"})}),
    lambda: "not base64!!",
    lambda: _zip_raw([(_symlink_info("plugin/silu_probe/link.py"), "/etc/passwd"), ("proposal.json", "{}")]),
])
def test_package_refusals(bad):
    with pytest.raises(GymError) as e:
        candidate_from_package(bad())
    assert e.value.code == "invalid_package"


def _symlink_info(name):
    info = zipfile.ZipInfo(name)
    info.external_attr = (0o120777 << 16)
    return info


def test_store_budget_reservations(tmp_path):
    from nexttransformer_b200.gym.store import Store
    s = Store(tmp_path / "s.sqlite", 100.0)
    s.open_job("j1", "q", 60.0)
    with pytest.raises(GymError) as e:
        s.open_job("j2", "q", 50.0)
    assert e.value.status == 402
    s.close_job("j1", "succeeded", 45.0)
    assert s.budget() == dict(limit=100.0, spent=45.0, reserved=0.0, available=55.0)
    s.open_job("j3", "q", 50.0)
    s.close_job("j3", "cancelled", 0.0)
    s.close_job("j3", "failed", 10.0)      # settling twice changes nothing
    assert s.budget()["spent"] == 45.0 and s.budget()["reserved"] == 0.0
    s.remember("k", "op", {"a": 1}, {"r": 1})
    assert s.remembered("k", "op", {"a": 1}) == {"r": 1}
    with pytest.raises(GymError):
        s.remembered("k", "op", {"a": 2})


SMI_XML = """<?xml version="1.0" ?><nvidia_smi_log>
<gpu id="00000000:18:00.0"><product_name>NVIDIA B200</product_name><uuid>GPU-aaa</uuid><minor_number>0</minor_number>
<fb_memory_usage><total>183359 MiB</total><used>0 MiB</used></fb_memory_usage><processes></processes></gpu>
<gpu id="00000000:2A:00.0"><product_name>NVIDIA B200</product_name><uuid>GPU-bbb</uuid><minor_number>1</minor_number>
<fb_memory_usage><total>183359 MiB</total><used>1024 MiB</used></fb_memory_usage>
<processes><process_info><pid>1</pid></process_info></processes></gpu></nvidia_smi_log>"""


def test_inventory_and_leases(tmp_path):
    from nexttransformer_b200.gym.resources import Leases, inventory
    gpus = inventory(lambda: SMI_XML)
    assert [g["index"] for g in gpus] == [0, 1] and gpus[1]["processes"] == 1
    assert gpus[0]["memory_total_mib"] == 183359 and gpus[0]["uuid"] == "GPU-aaa"
    assert inventory(lambda: (_ for _ in ()).throw(OSError("no driver"))) == []
    now = [1000.0]
    leases = Leases(tmp_path / "l.json", clock=lambda: now[0])
    assert leases.acquire([0, 1], "a", 10)
    assert not leases.acquire([1], "b", 10)          # all-or-nothing, held by a
    assert leases.free([0, 1]) == []
    now[0] += 11                                     # expired: reclaimed
    assert leases.acquire([1], "b", 10) and leases.free([0, 1]) == [0]
    leases.release("b")
    assert leases.free([0, 1]) == [0, 1]


def test_research_dp_equals_one_device():
    from nexttransformer_b200.gym.research import ResearchDP
    torch.manual_seed(0)
    net = torch.nn.Sequential(torch.nn.Linear(6, 16), torch.nn.Tanh(), torch.nn.Linear(16, 3))
    ref = copy.deepcopy(net)

    def loss_fn(m, x, y):
        return torch.nn.functional.cross_entropy(m(x), y)
    one = ResearchDP(ref, ["cpu"], lambda m: torch.optim.SGD(m.parameters(), lr=0.1))
    three = ResearchDP(net, ["cpu", "cpu", "cpu"], lambda m: torch.optim.SGD(m.parameters(), lr=0.1))
    assert three.shares(10) == [4, 3, 3]
    for step in range(3):
        g = torch.Generator().manual_seed(step)
        x, y = torch.randn(10, 6, generator=g), torch.randint(0, 3, (10,), generator=g)
        l1 = one.step(x, y, 4, loss_fn)
        l3 = three.step(x, y, 2, loss_fn)
        assert abs(l1 - l3) < 1e-5
    for a, b in zip(one.replicas[0].parameters(), three.replicas[2].parameters()):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)


@pytest.fixture
def gym(tmp_path):
    import uvicorn
    from nexttransformer_b200.gym.client import GymClient
    from nexttransformer_b200.gym.service import GymService, app
    service = GymService(tmp_path / "state", 1e12, gpus=[], smi_runner=lambda: SMI_XML, job_timeout=600)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    server = uvicorn.Server(uvicorn.Config(app(service, "tok"), host="127.0.0.1", port=port, log_level="error"))
    t = threading.Thread(target=server.run, daemon=True)
    t.start()
    for _ in range(100):
        if server.started:
            break
        time.sleep(0.05)
    yield GymClient(f"http://127.0.0.1:{port}", "tok"), service, port
    server.should_exit = True
    t.join(timeout=10)
    service.close()


def test_http_api_end_to_end(gym):
    import requests
    from nexttransformer_b200.gym.client import GymClient
    client, service, port = gym
    space = client.call("describe_space")
    assert "debug" in space["profiles"] and set(space["operation_schemas"]) == set(contract.OPERATIONS)
    with pytest.raises(GymError) as e:
        GymClient(client.endpoint, "wrong").call("get_budget")
    assert e.value.status == 401
    with pytest.raises(GymError) as e:
        client.call("no_such_op")
    assert e.value.status == 404
    with pytest.raises(GymError) as e:
        client.call("get_job")
    assert e.value.code == "invalid_params"
    r = requests.post(f"{client.endpoint}/v1/call", headers={"Authorization": "Bearer tok"},
                      json=dict(schema_version="v0", operation="get_budget"))
    assert r.status_code == 400

    pkg = make_package(_files())
    sub = client.call("submit_candidate", package_base64=pkg, idempotency_key="k1")
    again = client.call("submit_candidate", package_base64=pkg, idempotency_key="k1")
    assert sub == again and sub["method"] == "silu_probe"
    assert client.call("list_candidates")["items"][0]["candidate_id"] == sub["candidate_id"]
    cost = client.call("inspect_cost", candidate_id=sub["candidate_id"], profile_id="debug")
    assert cost["parameters"] > 0 and cost["flops_per_token"] > 0
    quote = client.call("quote_experiment", candidate_id=sub["candidate_id"], profile_id="debug", target_update=2)
    assert quote["affordable"] and quote["flops"] == pytest.approx(2 * cost["flops_per_update"])
    job = client.call("run_experiment", quote_id=quote["quote_id"], idempotency_key="run1")
    assert client.call("run_experiment", quote_id=quote["quote_id"], idempotency_key="run1")["job_id"] == job["job_id"]
    assert client.call("get_budget")["reserved"] == pytest.approx(quote["flops"])
    for _ in range(600):
        state = client.call("get_job", job_id=job["job_id"])["state"]
        if state in ("succeeded", "failed", "cancelled"):
            break
        time.sleep(0.5)
    res = client.call("get_result", job_id=job["job_id"])
    assert res["state"] == "succeeded", res
    assert len(res["result"]["losses"]) == 2 and res["result"]["devices"] == ["cpu"]
    budget = client.call("get_budget")
    assert budget["reserved"] == 0 and budget["spent"] == pytest.approx(res["spent_flops"]) and budget["spent"] > 0
    kinds = [e["kind"] for e in client.call("read_events")["items"]]
    assert kinds[0] == "candidate_submitted" and "job_succeeded" in kinds
    fin = client.call("finalize", candidate_id=sub["candidate_id"], profile_id="debug", idempotency_key="f")
    assert client.call("get_submission", submission_id=fin["submission_id"])["candidate_id"] == sub["candidate_id"]
    big = client.call("quote_experiment", candidate_id=sub["candidate_id"], profile_id="debug", target_update=99999)
    assert not big["affordable"]
    with pytest.raises(GymError) as e:
        client.call("run_experiment", quote_id=big["quote_id"])
    assert e.value.status == 402


def test_mcp_over_stdio(gym, tmp_path):
    client, service, port = gym
    cred = tmp_path / "cred.json"
    cred.write_text(json.dumps(dict(endpoint=client.endpoint, token="tok")))
    msgs = [dict(jsonrpc="2.0", id=1, method="initialize", params={}),
            dict(jsonrpc="2.0", method="notifications/initialized"),
            dict(jsonrpc="2.0", id=2, method="tools/list"),
            dict(jsonrpc="2.0", id=3, method="tools/call", params=dict(name="get_budget", arguments={})),
            dict(jsonrpc="2.0", id=4, method="tools/call", params=dict(name="get_job", arguments={"job_id": "x"}))]
    out = subprocess.run([sys.executable, "-m", "nexttransformer_b200.gym", "mcp", "--credential", str(cred)],
                         input="".join(json.dumps(m) + "\n" for m in msgs), capture_output=True, text=True,
                         timeout=120, check=True).stdout.splitlines()
    replies = {r["id"]: r for r in map(json.loads, out)}
    assert set(replies) == {1, 2, 3, 4}
    assert {t["name"] for t in replies[2]["result"]["tools"]} == set(contract.OPERATIONS)
    assert json.loads(replies[3]["result"]["content"][0]["text"])["limit"] == 1e12
    assert replies[4]["result"]["isError"]
