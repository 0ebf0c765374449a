"""Device completion protocol of the KV push (one GPU: sender and receiver share the device).

The signal kernel raises a flag word in stream order after the copies; the receiver's stream
waits for it with a bounded spin.  A flag that nothing raises makes the wait give up after its
limit, record its status and error word, and leave the context usable (no fault, no hang)."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C():
    from nanovllm_self_b200.ops._ext import load
    return load()


def test_signal_then_wait_passes(C):
    flags = torch.zeros(C.PUSH_FLAG_SLOTS, dtype=torch.int32, device="cuda")
    C.push_error(True)
    for epoch in (1, 2, 3):
        C.kv_push_signal(int(flags[5].data_ptr()), epoch)
        st = torch.zeros(1, dtype=torch.int32, device="cuda")
        C.kv_push_wait(int(flags[5].data_ptr()), epoch, int(1e9), st)
        torch.cuda.synchronize()
        assert st.item() == 1 and flags[5].item() == epoch
    # an older epoch is already reached
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.kv_push_wait(int(flags[5].data_ptr()), 2, int(1e9), st)
    torch.cuda.synchronize()
    assert st.item() == 1 and C.push_error(False) == 0


def test_wait_for_a_flag_nobody_raises_gives_up(C):
    flags = torch.zeros(C.PUSH_FLAG_SLOTS, dtype=torch.int32, device="cuda")
    C.push_error(True)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.time()
    C.kv_push_wait(int(flags[0].data_ptr()), 1, int(0.3e9), st)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    assert st.item() == 2
    assert C.push_error(True) == 210
    assert 0.25 < elapsed < 5.0
    x = torch.arange(8, device="cuda", dtype=torch.float32)
    assert float(x.sum().item()) == 28.0  # the context still runs work


def test_push_then_signal_orders_the_copy(C):
    """Copy, signal and wait in one stream (kernels that wait on each other never run as separate
    concurrent launches on one GPU here): after the wait the blocks are in place."""
    planes, nb, per = 4, 16, 4096
    src = torch.randn(2, planes // 2, nb, per, device="cuda").to(torch.bfloat16)
    dst = torch.zeros_like(src)
    flags = torch.zeros(C.PUSH_FLAG_SLOTS, dtype=torch.int32, device="cuda")
    ids_s = torch.tensor([3, 7, 1], dtype=torch.int32, device="cuda")
    ids_d = torch.tensor([0, 5, 9], dtype=torch.int32, device="cuda")
    C.comm_error(True)
    C.kv_push(src, ids_s, ids_d, int(dst.data_ptr()), nb)
    C.kv_push_signal(int(flags[1].data_ptr()), 1)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.kv_push_wait(int(flags[1].data_ptr()), 1, int(2e9), st)
    got = dst[:, :, ids_d.long()].clone()
    torch.cuda.synchronize()
    assert st.item() == 1 and C.comm_error(False) == 0
    assert torch.equal(got, src[:, :, ids_s.long()])
