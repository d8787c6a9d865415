"""The bounded wait of kh_decode_combine_from_peers, on one GPU.

The first call waits on a flag that nothing sets: after about a second the
kernel gives up, sets bit 2 of the device error word and writes zeros, and
the process keeps a usable context.  The second call finds its flags already
raised and must combine the records exactly like kh_decode_combine_strided."""
import pytest
import torch

from kudahitam import _lib, ops
from kudahitam import dist as khdist

pytestmark = pytest.mark.gpu


def test_peer_flag_wait_times_out_then_combines():
    D, R, world = 128, 4, 2
    g = torch.Generator(device="cuda").manual_seed(1)
    recs = torch.randn(world, R, D + 2, device="cuda", generator=g)
    recs[..., 1] = recs[..., 1].abs() + 0.5
    flags = torch.zeros(world, dtype=torch.int32, device="cuda")
    dv = ops._host_f32(torch.ones(D))
    out = torch.full((R, D), 7.0, device="cuda")
    _lib.call("kh_clear_device_error")
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    # epoch 1 never arrives: the wait must end by itself and report it
    _lib.call("kh_decode_combine_from_peers", recs.data_ptr(), flags.data_ptr(), 1, R, world, D,
              dv.data_ptr(), out.data_ptr(), stream)
    torch.cuda.synchronize()
    assert _lib.device_error() & 4
    assert torch.all(out == 0)
    # the checked form reports the timeout as an exception and clears the word
    with pytest.raises(khdist.PeerTimeoutError):
        khdist.check_peer_timeout()
    assert _lib.device_error() == 0
    khdist.check_peer_timeout()  # nothing pending: no exception
    # flags raised: the combine goes through and matches the strided combine
    flags.fill_(1)
    _lib.call("kh_decode_combine_from_peers", recs.data_ptr(), flags.data_ptr(), 1, R, world, D,
              dv.data_ptr(), out.data_ptr(), stream)
    want = ops.decode_combine_records(recs.transpose(0, 1), torch.ones(D),
                                      torch.empty(R, D, device="cuda"))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.allclose(out, want, rtol=1e-6, atol=1e-7)
