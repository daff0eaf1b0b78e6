"""Failure detection on the GPU without a GPU fault: a device-side bounded wait that
runs out ends the launch early with an error status the host reads, and the same
workspace keeps working afterwards.

Every wait in the tensor-core forward is bounded (default 2 s). Here the limit is set
to 200 microseconds and the test hook ptof_gdn_fwd_inject_stall makes the chain warp
first wait on a barrier that nothing arrives at, so waits give up on purpose (that
one, site 99, or another wait of the stalled CTA that runs out first): the kernel
raises its CTA abort flag, every
role runs out its loop without blocking, no further TMA load is issued, the loads and
UMMAs still in flight are drained and TMEM is released. Nothing traps, faults or
spins without a limit. The host then sees PTOF_ETIMEOUT from ptof_check_status (a
RuntimeError in Python); with the limit restored, the next launch on the same
workspace matches an untouched runner bit for bit.

The reference has no device-side wait limit; its nearest check is the determinism
gate (src/pto_fuser/gate.py:58-69), which two runs of a correct launch must pass.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_short_wait_limit_times_out_then_workspace_recovers():
    from pto_fuser import GDNChunkForward, make_gdn_inputs, native as nv
    B, H, T, D = 1, 4, 1024, 128
    inp = make_gdn_inputs(B, H, T, D, dtype=torch.bfloat16, device="cuda", seed=5)
    args = (inp["q"], inp["k"], inp["v"], inp["beta"], inp["g"])
    clean = GDNChunkForward(B, H, T, D, D)
    ref_o, ref_S = clean(*args)
    clean.check_status()

    run = GDNChunkForward(B, H, T, D, D)
    run.set_wait_limit(200_000)         # 200 us
    nv.check(nv.lib().ptof_gdn_fwd_inject_stall(run._ws, 1))
    run(*args)
    with pytest.raises(RuntimeError) as ei:
        run.check_status()
    assert isinstance(ei.value, nv.NativeError) and ei.value.code == nv.ETIMEOUT
    assert "gave up at site" in str(ei.value)

    # the context is usable and the status word was cleared by the read
    nv.check(nv.lib().ptof_gdn_fwd_inject_stall(run._ws, 0))
    run.set_wait_limit(2_000_000_000)
    o, S = run(*args)
    run.check_status()
    assert torch.equal(o, ref_o) and torch.equal(S, ref_S)
    run.close()
    clean.close()


def test_wait_limit_setter_rejects_zero_and_foreign_workspaces():
    from pto_fuser import native as nv
    L = nv.lib()
    assert L.ptof_ws_set_wait_limit(None, 1000) == nv.EINVAL
    ws = L.ptof_ws_setup()            # a generic workspace, not a forward's
    assert L.ptof_ws_set_wait_limit(ws, 1000) == nv.EINVAL
    L.ptof_ws_teardown(ws)
