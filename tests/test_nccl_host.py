"""The vocabulary-sharded exchange's host side (gs_nccl_create) against a fake NCCL library,
on CPU: a set-up that never completes returns GS_ETIMEOUT after its bound and aborts the
communicator, a failing set-up returns GS_ENCCL, a good one is created and destroyed."""
import nccl_util as NU


def test_comm_setup_timeout_error_and_success():
    lib = NU.build_fake_nccl()
    r = NU.run_worker(["host"], {"GS_NCCL_LIBRARY": lib})
    assert r.returncode == 0, r.stdout + r.stderr
    assert "host ok" in r.stdout
