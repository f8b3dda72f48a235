"""Single-GPU checks of the landing-buffer exchange primitives: a landing buffer from moe_peer_alloc seen as
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


def test_push_kernels_place_rows_like_pack_and_segment_sum():
    """moe_ep_push_pairs with destination blocks laid out in send order reproduces moe_ep_pack's
    rows and metadata exactly; moe_segment_sum_push with its output split over several
    destinations reproduces moe_segment_sum_rows exactly."""
    torch.manual_seed(3)
    T, k, E, G, H, C = 300, 4, 16, 4, 256, 2
    Tc = (T + C - 1) // C
    x = torch.randn(T, H, device="cuda").bfloat16()
    idx = torch.randint(0, E + 1, (T, k), device="cuda", dtype=torch.int32)  # E: skipped id
    w = torch.rand(T, k, device="cuda")
    groups, _ = candle_moe.ep_dest_groups(idx, E, G, Tc, C)
    zw = torch.zeros(groups.shape, device="cuda")
    off, p_tok, _, p_flat = candle_moe.route_prep_ex(groups, zw, C * G)
    U = int(off[C * G])
    rows_ref, meta_ref, _ = candle_moe.ep_pack(x, p_tok[:U], p_flat[:U], idx, w, E, G)
    rows = torch.zeros_like(rows_ref)
    meta = torch.zeros_like(meta_ref)
    offs = off.cpu().tolist()
    for c in range(C):
        rows_to = [rows.data_ptr() + offs[c * G + d] * H * 2 for d in range(G)]
        meta_to = [meta.data_ptr() + offs[c * G + d] * 2 * k * 4 for d in range(G)]
        candle_moe.ep_push_pairs(x, p_tok, p_flat, off, c, idx, w, E, G, rows_to, meta_to, None,
                                 _stream())
    torch.cuda.synchronize()
    assert torch.equal(rows, rows_ref)
    assert torch.equal(meta, meta_ref)

    n = 1000
    contrib = torch.randn(n, H, device="cuda").bfloat16()
    cuts = torch.sort(torch.randint(0, n + 1, (400,))).values
    start = torch.cat([torch.tensor([0]), cuts, torch.tensor([n])]).cuda()
    ref = candle_moe.segment_sum_rows(contrib, start)
    R = ref.shape[0]
    first = [0, 37, 37, 250, R]  # one origin gets no rows
    out = torch.zeros_like(ref)
    dst = [out.data_ptr() + first[s] * H * 2 for s in range(4)]
    candle_moe.segment_sum_push(contrib, start, dst, first, _stream())
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
