"""Suspension protocol, CUDA-checkpoint controller (fake backend) and the in-loop hook on 2 Gloo ranks.

Host-only fakes as in the reference's ``tests/test_training_suspend.py:14-36`` and
``tests/test_training_suspend_distributed.py``: no GPU is touched; failures are injected
in the fake ``cuda-checkpoint`` backend.
"""
import json
import multiprocessing as mp
import subprocess
import time
from pathlib import Path
from unittest.mock import Mock, patch

import pytest

from mimir_b200.train.suspension.controller import Controller, RestoreDeferred, wait_offloaded
from mimir_b200.train.suspension.protocol import atomic_write, claim, matches, read_json, steps, submit
from mimir_b200.train.suspension.supervisor import overrides, restart_command


class FakeCuda:
    def __init__(self, pids):
        self.states = dict.fromkeys(pids, "running")
        self.actions = []
        self.fail = None
        self.headroom = 100000

    def state(self, pid):
        return self.states[pid]

    def action(self, pid, action):
        self.actions.append((pid, action))
        if self.fail == (pid, action):
            raise RuntimeError("injected failure")
        self.states[pid] = {"lock": "locked", "checkpoint": "checkpointed", "restore": "locked",
                            "unlock": "running"}[action]

    def memory(self):
        return {(pid, "gpu0"): 32 for pid, s in self.states.items() if s != "checkpointed"}

    def free(self):
        return {"gpu0": self.headroom}


# ------------------------------------------------------------------------------- protocol
def test_queue_validation():
    assert steps("8 3 8") == [3, 8]
    for bad in ["-1", "0", "1.5", "foo", [True]]:
        with pytest.raises(ValueError):
            steps(bad)


def test_claim_does_not_delete_new_request(tmp_path):
    atomic_write(tmp_path / "launch.json", {})
    submit(tmp_path, [5, 2])
    submit(tmp_path, [3])
    old, values = claim(tmp_path)
    assert values == [2, 3, 5]
    submit(tmp_path, [10])
    old.unlink()
    assert claim(tmp_path)[1] == [10]


def test_submit_requires_launched_job(tmp_path):
    with pytest.raises(FileNotFoundError):
        submit(tmp_path, [1])


def test_invalid_request_is_quarantined(tmp_path):
    atomic_write(tmp_path / "suspend_after_steps", "oops")
    assert claim(tmp_path) == (None, [])
    assert len(list(tmp_path.glob("*.rejected.json"))) == 1


def test_generation_must_match():
    assert not matches({"job_id": "a", "step": 4, "generation": 1}, {"job_id": "a", "step": 4, "generation": 2})


# ------------------------------------------------------------------------------- controller
@pytest.fixture
def ctl(tmp_path):
    ranks = [{"rank": i, "pid": 100 + i, "start_ticks": str(i)} for i in range(2)]
    ready = {"job_id": "job", "generation": 1, "step": 7, "ranks": ranks}
    gen = tmp_path / "generation_000001"
    atomic_write(tmp_path / "launch.json", {"job_id": "job", "ranks": ranks})
    atomic_write(tmp_path / "suspend_ready.json", ready)
    for r in ranks:
        atomic_write(gen / f"ready.{r['pid']}.json", ready | r)
    backend = FakeCuda([100, 101])
    with patch("mimir_b200.train.suspension.controller.validate_process"):
        yield Controller(tmp_path, backend), backend, gen, ready, ranks


def test_success_order_and_idempotent_restore(ctl):
    c, b, gen, ready, _ = ctl
    c.offload()
    assert b.actions == [(100, "lock"), (101, "lock"), (100, "checkpoint"), (101, "checkpoint")]
    c.restore()
    n = len(b.actions)
    c.restore()
    assert len(b.actions) == n
    assert (gen / "resume.100").exists() and (gen / "resume.101").exists()
    atomic_write(c.root / "resumed.json", ready)
    with pytest.raises(RuntimeError, match="already resumed"):
        c.restore()


def test_partial_offload_recovers_without_false_admission(ctl):
    c, b, gen, _, _ = ctl
    b.fail = (101, "checkpoint")
    with pytest.raises(RuntimeError):
        c.offload()
    assert not (gen / "offloaded.json").exists()
    b.fail = None
    Controller(c.root, b).restore()
    assert set(b.states.values()) == {"running"}


def test_partial_restore_releases_no_rank(ctl):
    c, b, gen, _, _ = ctl
    c.offload()
    b.fail = (101, "restore")
    with pytest.raises(RuntimeError):
        c.restore()
    assert not list(gen.glob("resume.*"))
    b.fail = None
    b.headroom = 560  # room for the remaining 32 MiB plus margin, not for both ranks
    c.restore()
    assert len(list(gen.glob("resume.*"))) == 2


def test_memory_gate_and_user_hold(ctl):
    c, b, _, _, _ = ctl
    c.offload()
    b.headroom = 0
    with pytest.raises(RestoreDeferred, match="headroom"):
        c.restore()
    b.headroom = 100000
    (c.root / "hold").touch()
    with pytest.raises(RestoreDeferred, match="hold"):
        c.restore()


def test_missing_ready_rejects_before_gpu_operation(ctl):
    c, b, gen, _, _ = ctl
    (gen / "ready.101.json").unlink()
    with pytest.raises(FileNotFoundError):
        c.offload()
    assert b.actions == []


def test_cancel_before_offload(ctl):
    c, _, gen, _, _ = ctl
    c.cancel_unoffloaded()
    assert (gen / "resume.100").exists()
    with pytest.raises(RuntimeError, match="released"):
        c.offload()


def test_new_gpu_occupant_blocks_restore(ctl):
    c, b, gen, _, _ = ctl
    c.offload()
    with patch.object(b, "memory", return_value={(999, "gpu0"): 1}):
        with pytest.raises(RestoreDeferred, match="New GPU workload"):
            c.restore()
    assert not list(gen.glob("resume.*"))


def test_stale_process_rejects_before_gpu_operation(ctl):
    c, b, _, _, _ = ctl
    with patch("mimir_b200.train.suspension.controller.validate_process", side_effect=RuntimeError("stale")):
        with pytest.raises(RuntimeError, match="stale"):
            c.offload()
    assert b.actions == []


def test_cuda_error_output_is_journaled(ctl):
    c, b, gen, _, ranks = ctl
    error = subprocess.TimeoutExpired("checkpoint", 60, output=b"partial output", stderr=b"diagnostic")
    with patch.object(b, "action", side_effect=error):
        with pytest.raises(subprocess.TimeoutExpired):
            c.transition(gen, ranks[0], "checkpoint", "checkpointed")
    last = json.loads((gen / "operations.jsonl").read_text().splitlines()[-1])
    assert last["stderr"] == "diagnostic" and last["stdout"] == "partial output"


def test_pause_health_checks(ctl):
    c, b, gen, _, _ = ctl
    c.offload()
    wait_offloaded(Mock(poll=lambda: None), b, c, 0, float("inf"))
    assert json.loads((gen / "operations.jsonl").read_text().splitlines()[-1])["owned_gpu_mib"] == 0
    b.states[100] = "running"
    with pytest.raises(RuntimeError, match="Offloaded state changed"):
        wait_offloaded(Mock(poll=lambda: None), b, c, 0, float("inf"))
    b.states[100] = "checkpointed"
    with pytest.raises(RuntimeError, match="launcher exited"):
        wait_offloaded(Mock(poll=lambda: 1), b, c, 0, float("inf"))
    request = gen / "finish_early.request"
    request.touch()
    wait_offloaded(Mock(poll=lambda: None), b, c, 7200, float("inf"), request)
    c.restore()
    assert set(b.states.values()) == {"running"}


# ------------------------------------------------------------------------------- supervisor helpers
def test_overrides_replace_plus_keys():
    assert overrides(["a=1", "+b=2", "c=3"], {"b": 5, "a": 0}) == ["c=3", "b=5", "a=0"]


def test_restart_command_uses_published_checkpoint_and_remaining_steps(tmp_path):
    from mimir_b200.ckpt.contract import publish
    stage = tmp_path / "stage"
    stage.mkdir()
    atomic_write(stage / "checkpoint_state_step_4.json", {"step": 4, "carry_policy": "none"})
    publish(stage, tmp_path / "run" / "step_4", metadata={"mode": "exact", "tag": "step_4", "step": 4})
    root = tmp_path / "control"
    atomic_write(root / "queue.json", {"job_id": "j", "pending": [2, 8], "consumed": [4]})
    atomic_write(root / "suspend_after_steps", "12\n")
    ready = {"job_id": "j", "step": 4, "checkpoint": str(tmp_path / "run/step_4/checkpoint_state_step_4.json")}
    cmd = restart_command(["x=1", "suspend_after_steps=[4,8]"], root, ready)
    assert f"resume_checkpoint_path={tmp_path / 'run/step_4'}" in cmd
    assert "resume_checkpoint_tag=step_4" in cmd and "suspend_after_steps=[8,12]" in cmd and "x=1" in cmd


# ------------------------------------------------------------------------------- hook on 2 Gloo ranks
def _hook_worker(rank, root, rendezvous):
    import os
    os.environ["CUDA_VISIBLE_DEVICES"] = ""
    import torch
    import torch.distributed as dist
    from mimir_b200.train.suspension.runtime import SuspendHook
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"file://{rendezvous}", rank=rank, world_size=2)
    try:
        hook = SuspendHook(root, [2, 2], torch.device("cpu"), poll_steps=1, wait_seconds=0.02)
        totals = []
        for step in range(1, 7):
            v = torch.tensor(float(rank + step))
            dist.all_reduce(v)
            totals.append(v.item())
            hook.after_step(step, lambda: "cpu-test-checkpoint")
        atomic_write(Path(root) / f"result.{rank}.json", {"totals": totals, "queue": hook.queue,
                                                          "consumed": sorted(hook.consumed),
                                                          "generations": hook.generation})
    finally:
        dist.destroy_process_group()


def test_hook_two_ranks_late_requests_and_tokens(tmp_path):
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_hook_worker, args=(r, str(tmp_path), str(tmp_path / "rdv"))) for r in range(2)]
    for p in procs:
        p.start()
    deadline, released = time.monotonic() + 120, 0
    try:
        while any(p.is_alive() for p in procs):
            assert time.monotonic() < deadline, "ranks failed to resume"
            for path in tmp_path.glob("*/suspend_ready.json"):
                ready = read_json(path)
                gen = ready["generation"]
                if gen <= released:
                    continue
                assert len(ready["ranks"]) == 2
                assert ready["step"] == (2 if gen == 1 else 3)
                if gen == 1:
                    submit(path.parent, [1, 2, 3])  # one past, one consumed, one new
                for r in ready["ranks"]:
                    atomic_write(path.parent / f"generation_{gen:06d}" / f"resume.{r['pid']}", ready | r)
                released = gen
            time.sleep(0.02)
        for p in procs:
            p.join(10)
            assert p.exitcode == 0
        assert released == 2
        for r in range(2):
            res = read_json(tmp_path / f"result.{r}.json")
            assert res["totals"] == [3, 5, 7, 9, 11, 13]
            assert res["queue"] == [] and res["consumed"] == [1, 2, 3]
    finally:
        for p in procs:
            if p.is_alive():
                p.terminate()
            p.join(5)
