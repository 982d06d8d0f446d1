"""Chunk images of the tcgen05 NVFP4 decode kernel: every byte of an image is found again through the address rules
the kernel's header states (tile-major codes with the 128-byte swizzle, block scales in tcgen05.cp units), by plain
loops that share no code with the builder."""
import numpy as np
import torch

from luce_megakernel_b200 import nvfp4_images as I


def _rand_u8(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 256, shape, dtype=torch.uint8, generator=g)


def _check_image(img, rp, k, local_rows):
    """local_rows: {local row index: (codes row [k/2], scales row [k/16])}; everything else must be zero."""
    img = np.asarray(img)
    ncode = rp * (k // 2)
    codes = img[:ncode].reshape(k // 256, rp, 8, 16)
    sf = img[ncode:]
    seen_codes = np.zeros_like(codes, dtype=bool)
    seen_sf = np.zeros_like(sf, dtype=bool)
    for i, (crow, srow) in local_rows.items():
        for t in range(k // 256):
            for j in range(8):
                piece = crow[128 * t + 16 * j:128 * t + 16 * j + 16]
                assert np.array_equal(codes[t, i, j ^ (i % 8)], piece), (i, t, j)
                seen_codes[t, i, j ^ (i % 8)] = True
        for blk in range(k // 16):
            ks, b = blk // 4, blk % 4
            off = ks * 512 + (i % 32) * 16 + (i // 32) * 4 + b
            assert sf[off] == srow[blk], (i, blk)
            seen_sf[off] = True
    assert not codes[~seen_codes].any() and not sf[~seen_sf].any()


def test_phase_images_follow_the_stated_layout():
    for phase, n in (("dn_in", 8192), ("fa_in", 5120), ("out", 1024), ("down", 1024)):
        rp, k = I.PHASES[phase]
        packed, scales = _rand_u8((n, k // 2), 1), _rand_u8((n, k // 16), 2)
        imgs = I.build_phase_images(phase, packed, scales)
        nch = I.CHUNKS.get(phase, 1)
        assert imgs.reshape(I.IMAGE_CTAS, nch, -1).shape == (I.IMAGE_CTAS, nch, I.image_bytes(phase))
        imgs = imgs.reshape(I.IMAGE_CTAS, nch, -1)
        cut = I.split_rows(n)
        assert cut[0] == 0 and cut[-1] == n
        kc = k // nch
        for c in (0, 1, 73, 147):
            for q in range(nch):          # image q holds the q-th K part of the rows
                rows = {i: (packed[cut[c] + i, q * kc // 2:(q + 1) * kc // 2].numpy(),
                            scales[cut[c] + i, q * kc // 16:(q + 1) * kc // 16].numpy()) for i in range(cut[c + 1] - cut[c])}
                _check_image(imgs[c, q].numpy(), rp, kc, rows)


def test_gateup_images_pair_gate_and_up_rows():
    rp, k = I.PHASES["gateup"]
    gp, gs, up, us = _rand_u8((3584, 512), 3), _rand_u8((3584, 64), 4), _rand_u8((3584, 512), 5), _rand_u8((3584, 64), 6)
    imgs = I.build_gateup_images(gp, gs, up, us)
    assert imgs.shape == (I.IMAGE_CTAS, 36864)
    cut = I.split_rows(3584)
    for c in (0, 50, 147):
        rows = {}
        for i in range(cut[c + 1] - cut[c]):
            rows[i] = (gp[cut[c] + i].numpy(), gs[cut[c] + i].numpy())
            rows[I.UP_ROW0 + i] = (up[cut[c] + i].numpy(), us[cut[c] + i].numpy())
        _check_image(imgs[c].numpy(), rp, k, rows)


def test_lm_images_cover_every_row_once():
    vocab = 20011                       # not a multiple of anything
    packed, scales = _rand_u8((vocab, 512), 7), _rand_u8((vocab, 64), 8)
    imgs, chunks = I.build_lm_images(packed, scales)
    cut = I.split_rows(vocab)
    assert chunks == (max(cut[c + 1] - cut[c] for c in range(I.IMAGE_CTAS)) + 55) // 56
    assert imgs.shape == (I.IMAGE_CTAS, chunks, 36864)
    for c in (0, 99, 147):
        n = cut[c + 1] - cut[c]
        for q in range(chunks):
            rows = {i: (packed[cut[c] + 56 * q + i].numpy(), scales[cut[c] + 56 * q + i].numpy())
                    for i in range(max(0, min(56, n - 56 * q)))}
            _check_image(imgs[c, q].numpy(), 56, 1024, rows)


def test_image_sizes_match_the_kernel_constants():
    assert [I.image_bytes(p) for p in ("dn_in", "fa_in", "out", "gateup", "down", "lm")] == [36864, 28672, 24576, 36864, 21504, 36864]
