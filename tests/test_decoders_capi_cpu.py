"""Argument checks of the decoders' C-ABI entry points that answer before touching a GPU (runs without one): matrix
handles are views over placeholder addresses that are never dereferenced, since every call here is refused first."""
import ctypes

import pytest

FAKE = 1 << 20  # a 256-byte aligned placeholder "device" address; never dereferenced


def _view(C, out, inp):
    h = ctypes.c_void_p()
    C.check(C.lib().idol_b200_q8_view(ctypes.c_void_p(FAKE), None, out, inp, 0, ctypes.byref(h)))
    return h


def _oct_block(C, D=256, cond=16):
    h = ctypes.c_void_p()
    q, o, f1, f2 = _view(C, D, D), _view(C, D, D), _view(C, 4 * D, D), _view(C, D, 4 * D)
    C.check(C.lib().idol_b200_oct_block_create(q, o, f1, f2, ctypes.c_void_p(FAKE), ctypes.c_void_p(FAKE),
                                               ctypes.c_void_p(FAKE), None, cond, D // 64, ctypes.byref(h)))
    return h


def test_oct_block_and_decoder_shape_checks(pkg):
    C = pkg._capi
    L = C.lib()
    D = 256
    h = ctypes.c_void_p()
    # head_dim must be 64; cond_dim 1..64
    assert L.idol_b200_oct_block_create(_view(C, D, D), _view(C, D, D), _view(C, 4 * D, D), _view(C, D, 4 * D),
                                        ctypes.c_void_p(FAKE), ctypes.c_void_p(FAKE), ctypes.c_void_p(FAKE), None,
                                        16, 3, ctypes.byref(h)) == C.ERR_UNSUPPORTED
    assert L.idol_b200_oct_block_create(_view(C, D, D), _view(C, D, D), _view(C, 4 * D, D), _view(C, D, 4 * D),
                                        ctypes.c_void_p(FAKE), ctypes.c_void_p(FAKE), ctypes.c_void_p(FAKE), None,
                                        65, 4, ctypes.byref(h)) == C.ERR_UNSUPPORTED
    blk = _oct_block(C)
    arr = (ctypes.c_void_p * 1)(blk.value)
    dec = ctypes.c_void_p()
    args = [ctypes.cast(arr, ctypes.c_void_p), 1, ctypes.c_void_p(FAKE), None, _view(C, D, D), _view(C, D, 256),
            _view(C, D, D), _view(C, 6 * D, D)]
    # out_proj must have 8 outputs
    assert L.idol_b200_oct_decoder_create(*args, _view(C, 7, D), ctypes.c_void_p(FAKE), 42, ctypes.c_void_p(FAKE),
                                          4, ctypes.c_float(1e-6), ctypes.byref(dec)) == C.ERR_INVALID
    C.check(L.idol_b200_oct_decoder_create(*args, _view(C, 8, D), ctypes.c_void_p(FAKE), 42, ctypes.c_void_p(FAKE),
                                           4, ctypes.c_float(1e-6), ctypes.byref(dec)))
    ws = L.idol_b200_oct_decoder_workspace_bytes(dec, 1000, 500)
    assert ws > 1000 * D * 4
    pts = (ctypes.c_float * 30)()
    # refused before any device call: no condition for a decoder with blocks, empty condition, small workspace
    assert L.idol_b200_oct_sample_anchors(dec, None, 500, 10, 3, 1, pts, ctypes.c_void_p(FAKE), ws,
                                          None) == C.ERR_INVALID
    assert L.idol_b200_oct_sample_anchors(dec, ctypes.c_void_p(FAKE), 0, 10, 3, 1, pts, ctypes.c_void_p(FAKE), ws,
                                          None) == C.ERR_INVALID
    need = L.idol_b200_oct_decoder_workspace_bytes(dec, 10, 500)
    assert L.idol_b200_oct_sample_anchors(dec, ctypes.c_void_p(FAKE), 500, 10, 3, 1, pts, ctypes.c_void_p(FAKE),
                                          need - 256, None) == C.ERR_INVALID
    assert b"workspace" in L.idol_b200_last_error()
    L.idol_b200_oct_decoder_free(dec)
    L.idol_b200_oct_block_free(blk)


def test_gs_block_and_decoder_checks(pkg):
    C = pkg._capi
    L = C.lib()
    D = 256
    g = ctypes.c_void_p()
    vecs = [ctypes.c_void_p(FAKE)] * 6
    base = [_view(C, 3 * D, D), _view(C, D, D), _view(C, D, D), _view(C, D, D), _view(C, 4 * D, D),
            _view(C, D, 4 * D)]
    assert L.idol_b200_gs_block_create(*base, *vecs, ctypes.c_void_p(FAKE), None, 65, 4, ctypes.c_float(1e-6),
                                       ctypes.byref(g)) == C.ERR_UNSUPPORTED
    C.check(L.idol_b200_gs_block_create(*base, *vecs, ctypes.c_void_p(FAKE), None, 16, 4, ctypes.c_float(1e-6),
                                        ctypes.byref(g)))
    arr = (ctypes.c_void_p * 1)(g.value)
    dec = ctypes.c_void_p()
    rep = (ctypes.c_float * 9)(1.5, 0.0009, 0.004, 0.1, 1, 1, 1, 1, 0.1)
    # out_proj must hold 15 per_anchor rows
    assert L.idol_b200_gs_decoder_create(ctypes.cast(arr, ctypes.c_void_p), 1, ctypes.c_void_p(FAKE), None,
                                         _view(C, D, D), _view(C, 470, D), ctypes.c_void_p(FAKE), 42, 32,
                                         ctypes.c_void_p(FAKE), ctypes.c_float(-1.0), rep,
                                         ctypes.byref(dec)) == C.ERR_INVALID
    bad = (ctypes.c_float * 9)(1.5, 0.0009, 0.004, 1.5, 1, 1, 1, 1, 0.1)  # opacity bias outside (0, 1)
    assert L.idol_b200_gs_decoder_create(ctypes.cast(arr, ctypes.c_void_p), 1, ctypes.c_void_p(FAKE), None,
                                         _view(C, D, D), _view(C, 480, D), ctypes.c_void_p(FAKE), 42, 32,
                                         ctypes.c_void_p(FAKE), ctypes.c_float(-1.0), bad,
                                         ctypes.byref(dec)) == C.ERR_INVALID
    C.check(L.idol_b200_gs_decoder_create(ctypes.cast(arr, ctypes.c_void_p), 1, ctypes.c_void_p(FAKE), None,
                                          _view(C, D, D), _view(C, 480, D), ctypes.c_void_p(FAKE), 42, 32,
                                          ctypes.c_void_p(FAKE), ctypes.c_float(-1.0), rep, ctypes.byref(dec)))
    ws = L.idol_b200_gs_decoder_workspace_bytes(dec, 100, 200)
    assert L.idol_b200_gs_decoder_features(dec, ctypes.c_void_p(FAKE), 100, None, 200, ctypes.c_void_p(FAKE),
                                           ctypes.c_void_p(FAKE), ws, None) == C.ERR_INVALID
    assert L.idol_b200_gs_decoder_features(dec, ctypes.c_void_p(FAKE), 100, ctypes.c_void_p(FAKE), 200,
                                           ctypes.c_void_p(FAKE), ctypes.c_void_p(FAKE), ws - 256,
                                           None) == C.ERR_INVALID
    L.idol_b200_gs_decoder_free(dec)
    L.idol_b200_gs_block_free(g)


def test_gaussian_mlp_create_refuses_matrices_on_different_devices(pkg):
    C = pkg._capi
    L = C.lib()

    def view(out, inp, device):
        h = ctypes.c_void_p()
        C.check(L.idol_b200_q8_view(ctypes.c_void_p(FAKE), None, out, inp, device, ctypes.byref(h)))
        return h

    mlp = ctypes.c_void_p()
    for devs in ((0, 1, 0), (0, 0, 1)):
        assert L.idol_b200_gaussian_mlp_create(view(512, 128, devs[0]), view(512, 512, devs[1]),
                                               view(14, 512, devs[2]), ctypes.byref(mlp)) == C.ERR_INVALID
        assert b"different devices" in L.idol_b200_last_error()
        assert not mlp.value
    C.check(L.idol_b200_gaussian_mlp_create(view(512, 128, 0), view(512, 512, 0), view(14, 512, 0),
                                            ctypes.byref(mlp)))
    L.idol_b200_gaussian_mlp_free(mlp)


def test_int8_activation_gemm_refusals(pkg):
    C = pkg._capi
    L = C.lib()
    assert L.idol_b200_q8_gemm_int8act_workspace_bytes(10, 1024) >= 10 * 1024 + 2 * 10 * 32 * 4
    assert L.idol_b200_q8_gemm_int8act_workspace_bytes(10, 100) == -1
    w = _view(C, 256, 1024)
    ws = L.idol_b200_q8_gemm_int8act_workspace_bytes(10, 1024)
    args = lambda x_dtype, n_off, n, act, y_dtype, wsb: (w, ctypes.c_void_p(FAKE), x_dtype, 10, 1024, n_off, n, None,  # noqa: E731
                                                         0, act, ctypes.c_void_p(FAKE), y_dtype, 256,
                                                         ctypes.c_void_p(FAKE), wsb, None)
    assert L.idol_b200_q8_gemm_int8act(*args(C.F32, 0, 256, 0, C.F32, ws - 256)) == C.ERR_INVALID  # workspace
    assert b"workspace" in L.idol_b200_last_error()
    assert L.idol_b200_q8_gemm_int8act(*args(C.F32, 200, 100, 0, C.F32, ws)) == C.ERR_INVALID  # window past N
    assert L.idol_b200_q8_gemm_int8act(*args(C.F32, 0, 256, 9, C.F32, ws)) == C.ERR_INVALID  # activation
    assert L.idol_b200_q8_gemm_int8act(*args(C.F32, 0, 0, 0, C.F32, ws)) == C.OK  # empty window: nothing to do
