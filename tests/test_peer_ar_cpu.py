"""Host logic of PeerAllreduce's set-up on gloo ranks, with a fake of the
ftc_peer_ar_* entries: the IPC handles reach every rank in rank order, and a
rank whose allocation or mapping fails makes every rank raise the same error
(and free what it allocated) instead of leaving the others in a collective."""
import json
import os
import socket

import pytest

torch = pytest.importorskip("torch")


class FakeLib:
    """Stands in for libftcuda.so: records the calls, fails where told."""

    def __init__(self, rank, fail):
        self.rank, self.fail, self.log, self.err = rank, fail, [], b""

    def _rc(self, step):
        if self.fail.get(step) == self.rank:
            self.err = f"{step} refused on rank {self.rank}".encode()
            return 2
        return 0

    def ftc_peer_ar_create(self, rank, world, max_elems, out, handle):
        self.log.append(["create", rank, world, max_elems])
        rc = self._rc("create")
        if rc == 0:
            out._obj.value = 0x1000 + rank
            for i in range(len(handle)):
                handle[i] = (rank * 16 + i) & 0xFF
        return rc

    def ftc_peer_ar_open(self, ar, handles):
        self.log.append(["open", ar.value, bytes(handles).hex()])
        return self._rc("open")

    def ftc_peer_ar_destroy(self, ar):
        self.log.append(["destroy", ar.value])
        return 0

    def ftc_last_error(self):
        return self.err


def _rank_main(rank, world, port, out_dir, fail):
    import torch.distributed as dist
    from xwfes_b200 import ftc
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    fake = FakeLib(rank, fail)
    ftc._lib = fake
    res = {}
    try:
        ar = ftc.PeerAllreduce(4096)
        res["ok"] = True
        ar.close()
    except RuntimeError as e:
        res["error"] = str(e)
    finally:
        res["log"] = fake.log
        with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
            json.dump(res, f)
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(tmp_path, world, fail):
    import torch.multiprocessing as mp
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), fail), nprocs=world,
                       start_method="spawn", join=True)
    return [json.loads((tmp_path / f"r{r}.json").read_text()) for r in range(world)]


def _handle(rank, n=64):
    return bytes((rank * 16 + i) & 0xFF for i in range(n))


def test_handles_reach_every_rank_in_rank_order(tmp_path):
    res = _run(tmp_path, 3, {})
    allh = b"".join(_handle(r) for r in range(3)).hex()
    for r, x in enumerate(res):
        assert x.get("ok"), x
        assert x["log"] == [["create", r, 3, 4096], ["open", 0x1000 + r, allh],
                            ["destroy", 0x1000 + r]]


def test_a_failed_allocation_stops_every_rank(tmp_path):
    res = _run(tmp_path, 2, {"create": 1})
    for x in res:
        assert "ftc_peer_ar_create failed on rank(s) 1" in x["error"]
        assert "create refused on rank 1" in x["error"]
        assert not any(c[0] == "open" for c in x["log"])
    # rank 0 had allocated its buffer: it frees it; rank 1 has nothing to free
    assert res[0]["log"][-1] == ["destroy", 0x1000]
    assert [c[0] for c in res[1]["log"]] == ["create"]


def test_a_failed_mapping_stops_every_rank(tmp_path):
    res = _run(tmp_path, 2, {"open": 0})
    for r, x in enumerate(res):
        assert "ftc_peer_ar_open failed on rank(s) 0" in x["error"]
        assert [c[0] for c in x["log"]] == ["create", "open", "destroy"]


class RecordingLib:
    """Records the arguments of the fused GEMV entries."""

    def __init__(self):
        self.args = None

    def ftc_mul_mat_vec_silu(self, *a):
        self.args = a
        return 0

    def ftc_row_bytes(self, t, k):
        return (k // 256) * 144

    def ftc_last_error(self):
        return b""


def test_fused_silu_binding_passes_offsets_and_buffer(monkeypatch):
    from xwfes_b200 import formats as F, ftc
    rec = RecordingLib()
    monkeypatch.setattr(ftc, "_lib", rec)
    w = torch.zeros(64, dtype=torch.uint8)
    gu = torch.zeros((1, 2 * 512 + 64), dtype=torch.float32)
    y = torch.zeros((1, 8), dtype=torch.float32)
    ftc.mul_mat_vec_silu(w, F.Q4_K, 8, 512, gu, up_offset=576, y=y, stream=0)
    ar_, t, wp, n, k, rs, gp, off, yp, st = rec.args
    assert ar_ is None and t == F.Q4_K and (n, k, rs, off) == (8, 512, 288, 576)
    assert (wp, gp, yp) == (w.data_ptr(), gu.data_ptr(), y.data_ptr())
    ftc.mul_mat_vec_silu(w, F.Q4_K, 8, 512, gu, y=y, stream=0)
    assert rec.args[7] == 512  # up half right after the gate half by default

    class FakeAr:
        _ar = 0x1234

    ftc.mul_mat_vec_silu(w, F.Q4_K, 8, 512, gu, y=y, ar=FakeAr(), stream=0)
    assert rec.args[0] == 0x1234
