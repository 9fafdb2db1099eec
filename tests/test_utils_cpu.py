"""Fingerprints, guards, env validation, topology decisions and JSONL metrics (CPU)."""
import hashlib

import pytest
import torch

from bwn.config import tiny_qwen36
from bwn.models.qwen36 import build_qwen36
from bwn.parallel.topology import Topology, choose_comm_path
from bwn.utils import env, fingerprint as F
from bwn.utils.metrics import MetricsLog, read_jsonl


def test_gen_hash_format_matches_reference_definition():
    ids = [760, 6511, 314, 9338, 369]
    assert F.gen_hash(ids) == hashlib.md5(str(ids).encode()).hexdigest()[:12]
    assert F.gen_hash(torch.tensor(ids)) == F.gen_hash(ids)


def test_logits_fingerprint():
    x = torch.zeros(2, 10)
    x[0, 7] = 3.0
    x[0, 2] = 2.0
    fp = F.logits_fingerprint(x)
    assert fp["top5"][:2] == [7, 2] and fp["finite"] and fp["sum"] == 5.0
    x[1, 1] = float("nan")
    assert not F.logits_fingerprint(x)["finite"]


def test_assert_disjoint_catches_overlap_allows_slices():
    base = torch.zeros(4, 8)
    F.assert_disjoint([base[i] for i in range(4)])           # per-layer slices: disjoint
    with pytest.raises(RuntimeError, match="overlap"):
        F.assert_disjoint([base[0:2], base[1:3]])             # overlapping views
    with pytest.raises(RuntimeError, match="overlap"):
        F.assert_disjoint([base, base.view(-1)])               # same memory, two views
    F.assert_disjoint([base[:, :4], torch.zeros(3)])


def test_occupancy_gate_fires_on_an_empty_layer(monkeypatch):
    st = torch.ones(3, 2, 4)
    assert F.assert_occupancy(st, "x") == [2, 2, 2]
    st[1] = 0
    with pytest.raises(RuntimeError, match=r"layers \[1\]"):
        F.assert_occupancy(st, "x")
    monkeypatch.setenv("BWN_OCCUPANCY_CHECK", "0")
    assert F.assert_occupancy(st, "x") == []


def test_qwen36_state_guards_after_decode():
    cfg = tiny_qwen36(layers=4)
    m = build_qwen36(cfg, device="cpu", dtype=torch.float32)
    st = m.new_state(2, 16)
    with pytest.raises(RuntimeError):   # nothing written yet
        F.check_qwen36_state(st)
    ids = torch.tensor([[3, 4, 5], [6, 7, 8]])
    m.prefill(ids, st)
    rows = F.check_qwen36_state(st)
    assert all(n > 0 for n in rows["ssm"]) and all(n > 0 for n in rows["k"])


def test_env_validation(monkeypatch):
    assert env.validate({})["BWN_PDL"] == 1
    with pytest.raises(ValueError, match="unknown"):
        env.validate({"BWN_NOPE": "1"})
    with pytest.raises(ValueError, match="expected one of"):
        env.validate({"BWN_FUSED_COMM": "maybe"})
    with pytest.raises(ValueError, match="cannot be combined"):
        env.validate({"BWN_NO_REDUCE": "1", "BWN_FUSED_COMM": "on"})
    monkeypatch.setenv("BWN_PROFILE_STEPS", "7")
    assert env.get("BWN_PROFILE_STEPS") == 7
    assert "BWN_PDL" in env.describe()


def test_choose_comm_path():
    full = Topology(8, ["B200"] * 8, [[True] * 8 for _ in range(8)], multicast=True)
    assert choose_comm_path(full, 1) == "single"
    assert choose_comm_path(full, 8) == "fused_nvls"
    assert choose_comm_path(full, 8, "off") == "nccl"
    nomc = Topology(8, ["B200"] * 8, [[True] * 8 for _ in range(8)], multicast=False)
    assert choose_comm_path(nomc, 4) == "fused_p2p"
    broken = Topology(2, ["B200"] * 2, [[True, False], [False, True]], multicast=True)
    assert choose_comm_path(broken, 2) == "nccl"
    with pytest.raises(RuntimeError):
        choose_comm_path(broken, 2, "on")


def test_metrics_jsonl(tmp_path):
    p = str(tmp_path / "m" / "run.jsonl")
    log = MetricsLog(p, None, run={"model": "tiny"})
    log.timing("decode_step", 1.25, batch=4)
    recs = read_jsonl(p)
    assert [r["event"] for r in recs] == ["run", "decode_step"]
    assert recs[1]["ms"] == 1.25 and recs[1]["batch"] == 4 and recs[0]["model"] == "tiny"


def test_symm_canary_registry_reports_a_changed_tail():
    """The guard-tail registry without symmetric memory: a stand-in buffer
    registered as an allocation is reported once its tail changes, and dropped
    once it is freed."""
    import weakref

    from bwn.parallel import symm
    full = torch.empty(100 + symm.CANARY_BYTES, dtype=torch.uint8)
    full[:100].zero_()
    full[100:].fill_(symm.CANARY)
    symm._guarded.append((weakref.ref(full), 100, "standin"))
    full[:100].fill_(7)  # writes inside the region are fine
    assert "standin" not in symm.check_canaries()
    full[100 + 5] = 0    # one byte past the end
    assert "standin" in symm.check_canaries()
    del full
    assert "standin" not in symm.check_canaries()
    assert all(name != "standin" for _, _, name in symm._guarded)


def test_every_layer_state_changes_every_step():
    from bwn.config import tiny_qwen36
    from bwn.models.qwen36 import build_qwen36
    from bwn.utils import fingerprint as F
    cfg = tiny_qwen36()
    m = build_qwen36(cfg, seed=2, dtype=torch.float32)
    st = m.new_state(2, 16)
    tok = torch.tensor([3, 7], dtype=torch.int32)
    for _ in range(3):
        snap = F.snapshot_state(st)
        tok = m.decode_step(tok, st).int()
        F.assert_state_advanced(snap, st)
    snap = F.snapshot_state(st)
    st.positions.add_(1)  # a step that wrote nothing
    with pytest.raises(RuntimeError, match="was not written"):
        F.assert_state_advanced(snap, st)


def test_single_domain_check(monkeypatch):
    """Fused peer-memory paths refuse a group whose ranks sit on different hosts."""
    from bwn.parallel import topology as T
    from bwn.parallel.comm import Comm
    assert len(T.hosts_of(Comm.single())) == 1
    monkeypatch.setattr(T, "hosts_of", lambda comm: ["node-a", "node-a"])
    T.require_single_domain(Comm(None, 0, 2), "x")  # one host: fine
    monkeypatch.setattr(T, "hosts_of", lambda comm: ["node-a", "node-b"])
    with pytest.raises(RuntimeError, match="spans hosts"):
        T.require_single_domain(Comm(None, 0, 2), "fused comm")


def test_clock_summary_parsing():
    from bwn.utils.clocks import ClockSampler
    c = ClockSampler()
    c.lines = ["0, 1860, 1965, 900.1, 0x0, Not Active, Not Active, Not Active, Not Active",
               "0, 1320, 1965, 999.9, 0x4, Not Active, Not Active, Not Active, Active",
               "garbage", "0, N/A, 1965, 1, 0, a, b, c, d"]
    s = c.summary()
    assert s["samples"] == 2 and s["sm_mhz"] == (1860 + 1320) / 2 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"] and "suspect" not in s  # power cap: kept and noted
    c.lines = ["0, 1500, 1965, 700, 0x40, Not Active, Active, Not Active, Not Active"]
    assert c.summary()["suspect"].startswith("throttled: hw_thermal_slowdown")
    c.lines = ["0, 1000, 1965, 400, 0x0, Not Active, Not Active, Not Active, Not Active"]
    assert "held below max" in c.summary()["suspect"]
    c.lines = []
    assert c.summary()["samples"] == 0
