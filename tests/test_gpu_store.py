"""The CPU tier's pinned slab pool and disk prefetch on a CUDA host."""

import pytest
import torch

from polylora_b200.store import PinnedSlabPool

pytestmark = pytest.mark.gpu


def test_pinned_slab_is_reused_only_after_its_copy_completes():
    pool = PinnedSlabPool(1 << 18, slabs_per_arena=2)
    a, b = pool.acquire(), pool.acquire()
    assert a.is_pinned() and b.is_pinned() and a.numel() == 1 << 18
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        torch.cuda._sleep(100_000_000)  # bounded busy kernel standing in for a long copy
        ev = torch.cuda.Event()
        ev.record(side)
    pool.note_use(a, ev)
    pool.release(a)
    assert len(pool.retired) == 1 and not pool.free  # its copy may still read it
    c = pool.acquire()  # a fresh arena, not the retired slab
    assert c.data_ptr() not in (a.data_ptr(), b.data_ptr()) and len(pool.arenas) == 2
    ev.synchronize()
    pool.release(b)
    pool.release(c)
    got = {pool.acquire().data_ptr() for _ in range(4)}
    assert a.data_ptr() in got  # reclaimed once its event completed


def test_slot_fill_rejects_records_outside_the_image(native):
    """plora_slot_fill reads only blocks inside the image: a record whose B
    block runs past image_bytes fills the slot as rank 0 and raises
    PLORA_DEV_IMAGE_RANGE; a valid record is transposed into the slot.  The
    staging buffer is much larger than the image, so even an unchecked read of
    the bad record would stay inside it."""
    import ctypes

    dev = torch.device("cuda")
    ns, R, K, N, r = 3, 4, 8, 6, 2
    A = torch.full((ns, K, R), 7.0, device=dev)
    B = torch.full((ns, R, N), 7.0, device=dev)
    ranks = torch.full((ns,), 9, dtype=torch.int32, device=dev)
    scales = torch.full((ns,), 9.0, device=dev)
    mods = (native.SlotModule * 1)()
    mods[0].lora_a, mods[0].lora_b = A.data_ptr(), B.data_ptr()
    mods[0].ranks, mods[0].scales = ranks.data_ptr(), scales.data_ptr()
    mods[0].in_features, mods[0].out_features = K, N
    table = torch.frombuffer(bytearray(bytes(mods)), dtype=torch.uint8).to(dev)
    a_blk = torch.arange(r * K, dtype=torch.float32).reshape(r, K)  # PEFT lora_A (rank, in)
    b_blk = torch.arange(N * r, dtype=torch.float32).reshape(N, r) + 100  # PEFT lora_B (out, rank)
    staging = torch.empty(1 << 16, dtype=torch.uint8, device=dev)

    def fill(slot, b_offset):
        img = torch.zeros(768, dtype=torch.uint8)
        rec = native.SlotRecord(a_offset=256, b_offset=b_offset, rank=r, scale=0.5)
        img[: ctypes.sizeof(rec)] = torch.frombuffer(bytearray(bytes(rec)), dtype=torch.uint8)
        img[256:256 + 4 * r * K] = a_blk.view(torch.uint8).flatten()
        if b_offset + 4 * N * r <= img.numel():
            img[b_offset:b_offset + 4 * N * r] = b_blk.view(torch.uint8).flatten()
        img = img.pin_memory()
        native.call("plora_slot_fill", table.data_ptr(), 1, slot, ns, R, native.DTYPE_F32, img.data_ptr(),
                    img.numel(), staging.data_ptr(), staging.numel(), torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()

    native.device_status(clear=True)
    fill(1, 512)
    assert native.device_status(clear=True) == 0
    want_a = torch.zeros(K, R)
    want_a[:, :r] = a_blk.t()
    want_b = torch.zeros(R, N)
    want_b[:r] = b_blk.t()
    assert torch.equal(A[1].cpu(), want_a) and torch.equal(B[1].cpu(), want_b)
    assert int(ranks[1]) == r and float(scales[1]) == 0.5
    fill(2, 736)  # B block = bytes 736..784 of a 768-byte image
    assert native.device_status(clear=True) & native.DEV_IMAGE_RANGE
    assert not A[2].any() and not B[2].any() and int(ranks[2]) == 0 and float(scales[2]) == 0.0
    assert bool((A[0] == 7.0).all()) and int(ranks[0]) == 9  # other slots untouched
