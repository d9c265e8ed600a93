"""CPU oracle for the block-sparse masked attention path — TEST INFRASTRUCTURE ONLY.

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline / `--impl reference` legs
may import this package, and only as the checker or as the timed CPU stand-in for the reference's
own CPU path. The product (`faster_weathernext` and `libfwn_attn.so`) never calls into it.

It restates, in NumPy, the reference's (Raymondlol/Faster-WeatherNext v0.2.0) algorithms:

* `tiles`     — `build_tile_mask` (src/faster_weathernext/pallas_attn.py:85-109), `hilbert_order` and
                `_hilbert3` (pallas_attn.py:41-82), `build_chunked_mask` (src/faster_weathernext/patch.py:106-127),
                plus the 128-row pairing the CUDA kernels walk (derived from the 64x32 list).
* `attention` — the XLA chunked attention path (patch.py:130-162: einsum * scale, where(mask, ., -1e30),
                softmax, einsum), the forward's log-sum-exp (pallas_attn.py:138-140), and the analytic
                float64 gradient of the reference's kernel tests (tests/test_pallas_kernel.py:15-21, 58-69).

Parity is pinned: `tests/golden/make_golden.py` runs the reference's own NumPy functions (the tile
builder, the Hilbert order, the chunked-mask builder and the float64 test references) in the
build container and stores their outputs in `tests/golden/`; `tests/test_oracle_golden.py` checks
this package against them.
"""
