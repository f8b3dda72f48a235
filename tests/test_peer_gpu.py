"""Single-GPU checks of the p2p exchange primitives: a landing buffer from moe_peer_alloc seen as
a tensor, copy-engine copies into it, arrival flags set by moe_peer_signal and awaited by
moe_peer_wait, and the bounded wait: a flag that nothing sets ends the wait after its limit with
the ERR_PEER_WAIT bit in the device error word, and the stream (and context) stay usable."""
import pytest
import torch

import candle_moe

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream()


def test_landing_buffer_copy_signal_wait():
    candle_moe.device_error_bits(0, clear=True)
    nbytes = 1 << 20
    addr, handle = candle_moe.peer_alloc(nbytes, 0)
    buf = None
    try:
        assert len(handle) == candle_moe.PEER_HANDLE_BYTES
        buf = candle_moe.device_bytes(addr, nbytes, 0)
        assert buf.is_cuda and buf.numel() == nbytes and int(buf.sum()) == 0  # zero-filled
        src = torch.randint(0, 256, (4096,), dtype=torch.uint8, device="cuda")
        candle_moe.copy_async(addr + 256, src.data_ptr(), src.numel(), _stream())
        # flags 0..3 at the start of the buffer; signal them to 7, then wait for 7 and for 5
        candle_moe.peer_signal([addr + 4 * i for i in range(4)], 7, _stream())
        candle_moe.peer_wait(addr, 4, 7, 1.0, _stream())
        candle_moe.peer_wait(addr, 4, 5, 1.0, _stream())
        torch.cuda.synchronize()
        assert torch.equal(buf[256:256 + 4096], src)
        assert buf[:16].view(torch.int32).tolist() == [7, 7, 7, 7]
        assert candle_moe.device_error_bits(0) == 0
    finally:
        del buf
        candle_moe.peer_free(addr, 0)


def test_wait_on_a_flag_nobody_sets_times_out_with_error_bit():
    candle_moe.device_error_bits(0, clear=True)
    addr, _ = candle_moe.peer_alloc(4096, 0)
    try:
        candle_moe.peer_wait(addr, 2, 1, 0.05, _stream())  # flags stay 0: runs out after 50 ms
        x = torch.ones(8, device="cuda")
        y = (x * 2).sum()  # the stream continues after the wait gave up
        torch.cuda.synchronize()
        assert float(y) == 16.0
        bits = candle_moe.device_error_bits(0, clear=True)
        assert bits & candle_moe.ERR_PEER_WAIT, bits
        assert candle_moe.device_error_bits(0) == 0
    finally:
        candle_moe.peer_free(addr, 0)
