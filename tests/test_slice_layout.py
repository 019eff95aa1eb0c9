"""The frame kernel's per-CTA slice layout of its weight matrices (k_slice_layout in
navi-tts_b200/csrc/frame.cu, layout described in frame_kernel.cuh): row r of an R x K
matrix belongs to CTA b with floor(R b / G) <= r < floor(R (b+1) / G); inside that CTA's
byte range [r0 K, r1 K) element (r, k) moves to ((k/8)(r1-r0) + (r-r0)) 8 + k%8.  The
mapping must be a bijection that never leaves the CTA's range (the producer streams exactly
that range) -- checked here for the shapes the benchmark and tests use."""
import numpy as np
import pytest


def owner(r, R, G):
    return ((r + 1) * G + R - 1) // R - 1


def split(R, b, G):
    return (R * b) // G, (R * (b + 1)) // G


@pytest.mark.parametrize("R,K", [(4096, 1024), (1024, 2048), (3072, 1024), (1024, 3072), (2048, 1024), (1024, 256), (512, 256),
                                 (256, 512), (7, 64)])
@pytest.mark.parametrize("G", [148, 132, 7, 1])
def test_slice_layout_is_a_bijection_within_each_cta(R, K, G):
    nk = K // 8
    r = np.arange(R)[:, None]
    kc = np.arange(nk)[None, :]
    b = owner(r, R, G)
    r0 = (R * b) // G
    r1 = (R * (b + 1)) // G
    assert np.all((r0 <= r) & (r < r1))
    dst = r0 * K + (kc * (r1 - r0) + (r - r0)) * 8
    flat = np.sort(dst.ravel())
    assert np.array_equal(flat, np.arange(0, R * K, 8))           # every 16-byte slot exactly once
    assert np.all(dst >= r0 * K) and np.all(dst + 8 <= r1 * K)    # inside the CTA's streamed range
