"""Per-CTA chunk images of tensor-scale NVFP4 weights for the tcgen05 decode kernel (mk_decode_nvfp4_mma).

The decode megakernel gives every CTA a fixed share of the rows of each projection phase (rows [n c / G, n (c + 1) / G)
of the phase's n rows for CTA c of G).  The mma.sync variants stream those rows as they lie in the quantised matrices;
the tcgen05 variant wants them in the shared-memory layout the tensor core reads, so they are rearranged once, here,
into one image per (phase, CTA): a phase is then a single bulk copy per CTA.  The reference packs its NVFP4 weights
on the host in the same spirit (megakernel/model_nvfp4.py:249-337), for its own kernel's access pattern.

Image of a phase with K input features and RP padded rows (RP = 56 qkv|z, gate|up and LM-head chunks, 40 q|k|v,
8 out / down projections; the down projection is cut into two images of K = 1792 each, k-tiles 0-6 and 7-13):

  codes  : K / 256 tiles of RP x 128 bytes.  Tile t, local row i holds the 256 e2m1 codes k = 256 t .. 256 t + 255 of
           the row (two per byte, even k in the low nibble), its eight 16-byte pieces stored at piece j ^ (i % 8):
           the 128-byte swizzle of a K-major tcgen05 operand.  Rows past the CTA's share are zero.
  scales : one unit of 512 bytes = 32 lanes x 16 bytes per MMA step of 64 k, the shape one tcgen05.cp (32x128b,
           warpx4) moves into four tensor-memory columns: unit ks, lane l, byte 4 g + b = the scale of block b
           (k = 64 ks + 16 b ..) of local row l + 32 g; bytes of rows the image does not have are zero.

gate|up images keep gate row o at local row o - first and the up row of the same output at local row 28 + o - first.
The LM head has one image per (CTA, 56-row chunk of the CTA's share).
"""
import torch

IMAGE_CTAS = 148                # the decode grid the images are cut for: one CTA per SM of a B200

PHASES = {                      # name -> (padded rows, K)
    "dn_in": (56, 1024), "fa_in": (40, 1024), "out": (8, 2048), "gateup": (56, 1024), "down": (8, 3584),
    "lm": (56, 1024),
}
CHUNKS = {"down": 2}            # images per CTA (K halves); 1 for every other layer phase
UP_ROW0 = 28                    # local row of the first up-projection row in a gate|up image


def image_bytes(phase):
    rp, k = PHASES[phase]
    k //= CHUNKS.get(phase, 1)
    return rp * (k // 2) + (k // 64) * 512


def split_rows(n, ctas=IMAGE_CTAS):
    """First row of every CTA's share (ctas + 1 entries), the kernel's n * c / G."""
    return [(n * c) // ctas for c in range(ctas + 1)]


def _gather_rows(mat, idx):
    """mat [R, W] uint8, idx [..] int64 with -1 for padding -> [.., W], zero rows where idx < 0."""
    out = mat[idx.clamp(min=0)]
    out[idx < 0] = 0
    return out


def _swizzle_codes(rows):
    """[G, RP, K/2] -> [G, (K/256) * RP * 128]: tile-major, 16-byte pieces XOR-swizzled by the row index."""
    G, RP, KB = rows.shape
    T = KB // 128
    x = rows.reshape(G, RP, T, 8, 16)
    i = torch.arange(RP, device=rows.device) % 8
    j = torch.arange(8, device=rows.device)
    src = (j[None, :] ^ i[:, None])                       # output piece j takes input piece j ^ (i % 8)
    x = torch.gather(x, 3, src[None, :, None, :, None].expand(G, RP, T, 8, 16))
    return x.permute(0, 2, 1, 3, 4).reshape(G, T * RP * 128)


def _scale_units(sc, rp):
    """sc [G, 32 or 64, K/16] block scales of the local rows -> [G, units * 512] in tcgen05.cp order."""
    G, R, NB = sc.shape
    ks = NB // 4
    groups = R // 32
    x = sc.reshape(G, groups, 32, ks, 4).permute(0, 3, 2, 1, 4)          # [G, step, lane, group, block]
    out = torch.zeros(G, ks, 32, 4, 4, dtype=sc.dtype, device=sc.device)
    out[:, :, :, :groups] = x
    return out.reshape(G, -1)


def _local_index(first, count, rp, device):
    """[G, rp] row indices first[c] + i for i < count[c], else -1."""
    i = torch.arange(rp, device=device)[None, :]
    idx = first[:, None] + i
    return torch.where(i < count[:, None], idx, torch.full_like(idx, -1))


def build_phase_images(phase, packed, scales, ctas=IMAGE_CTAS):
    """packed [n, K/2] uint8, scales [n, K/16] uint8 (rows of all the phase's matrices concatenated in kernel row
    order) -> uint8 [ctas, image_bytes(phase)]."""
    rp, k = PHASES[phase]
    n = packed.shape[0]
    assert packed.shape[1] == k // 2 and scales.shape == (n, k // 16)
    dev = packed.device
    cut = torch.tensor(split_rows(n, ctas), device=dev, dtype=torch.int64)
    first, count = cut[:-1], cut[1:] - cut[:-1]
    if int(count.max()) > rp:
        raise ValueError(f"{phase}: a CTA owns {int(count.max())} rows, the image holds {rp}")
    sr = 32 if rp <= 32 else 64
    codes = _swizzle_codes(_gather_rows(packed, _local_index(first, count, rp, dev)))
    sf = _scale_units(_gather_rows(scales, _local_index(first, count, sr, dev)), rp)
    nch = CHUNKS.get(phase, 1)
    if nch == 1:
        return torch.cat([codes, sf], dim=1).contiguous()
    # K halves: image q holds k-tiles and scale units of its half; [ctas, nch, image_bytes]
    codes = codes.reshape(ctas, nch, -1)
    sf = sf.reshape(ctas, nch, -1)
    return torch.cat([codes, sf], dim=2).contiguous()


def build_gateup_images(gate_packed, gate_scales, up_packed, up_scales, ctas=IMAGE_CTAS):
    """gate / up [3584, 512] codes and [3584, 64] scales -> uint8 [ctas, image_bytes('gateup')]."""
    rp, k = PHASES["gateup"]
    n = gate_packed.shape[0]
    dev = gate_packed.device
    cut = torch.tensor(split_rows(n, ctas), device=dev, dtype=torch.int64)
    first, count = cut[:-1], cut[1:] - cut[:-1]
    if int(count.max()) > UP_ROW0:
        raise ValueError(f"gate|up: a CTA owns more than {UP_ROW0} outputs")
    idx = _local_index(first, count, UP_ROW0, dev)
    pad = torch.full((ctas, 64 - 2 * UP_ROW0), -1, dtype=torch.int64, device=dev)
    codes = _swizzle_codes(torch.cat([_gather_rows(gate_packed, idx), _gather_rows(up_packed, idx)], dim=1))
    sf = _scale_units(torch.cat([_gather_rows(gate_scales, idx), _gather_rows(up_scales, idx),
                                 _gather_rows(up_scales, pad)], dim=1), rp)
    return torch.cat([codes, sf], dim=1).contiguous()


def build_lm_images(packed, scales, ctas=IMAGE_CTAS):
    """LM head [vocab, 512] codes and [vocab, 64] scales -> (uint8 [ctas, chunks, image_bytes('lm')], chunks)."""
    rp, k = PHASES["lm"]
    n = packed.shape[0]
    dev = packed.device
    cut = torch.tensor(split_rows(n, ctas), device=dev, dtype=torch.int64)
    first, count = cut[:-1], cut[1:] - cut[:-1]
    chunks = (int(count.max()) + rp - 1) // rp
    q = torch.arange(chunks, device=dev, dtype=torch.int64)
    f = (first[:, None] + rp * q[None, :]).reshape(-1)
    cnt = (count[:, None] - rp * q[None, :]).clamp(min=0, max=rp).reshape(-1)
    codes = _swizzle_codes(_gather_rows(packed, _local_index(f, cnt, rp, dev)))
    sf = _scale_units(_gather_rows(scales, _local_index(f, cnt, 64, dev)), rp)
    return torch.cat([codes, sf], dim=1).reshape(ctas, chunks, -1).contiguous(), chunks
