"""CPU checks of the GE TransData-level entry points against GE's own tests.

Every TransFormat / TransShape / TransDataFormat expectation in GE's
format_transfer_fractal_nz_unittest.cc, format_transfer_fractal_zz_unittest.cc and
format_transfer_transpose_unittest.cc whose outcome is decided before any data
moves (all failures, all TransShape calls) is replayed through the C ABI here;
the data-moving successes run in the GPU tests.  The status classes map onto GE's codes through dcopy_status_to_ge.
"""
import numpy as np
import pytest

import ge_goldens

CLASS = {"FormatTransferFractalNz": 1, "FormatTransferFractalNzND": 2,
         "FormatTransferTranspose": 3, "FormatTransferFractalZz": 4,
         "FormatTransferFractalZzND": 5, "FormatTransferFractalZ": 6,
         "FormatTransferFractalZTbe": 7, "FormatTransferFracZNchw": 8,
         "FormatTransferFracZHwcn": 9, "FormatTransferFracZNhwc": 10}


def _fmt(name):
    return ge_goldens.FMT[name]


def _dt(name):
    return ge_goldens.DT[name]


def _status(dcopy, fn, *args, **kw):
    try:
        fn(*args, **kw)
        return 0
    except dcopy.DcopyError as e:
        return dcopy.status_to_ge(e.code)


@pytest.mark.parametrize("which", ["nz", "zz", "transpose"])
def test_ge_expectations_decided_on_host(dcopy, reference_root, which):
    checked = 0
    for case in ge_goldens.load(reference_root, which):
        for e in case.expects:
            a = case.args.get(e.args) if e.args else None
            if e.call == "TransShape" and a is not None:
                got = _status(dcopy, dcopy.trans_shape, CLASS[e.transfer_class],
                              _fmt(a.src_format), a.src_shape, _dt(a.dtype), _fmt(a.dst_format),
                              a.c0[1] if len(a.c0) > 1 else 16)
            elif e.call == "TransShape":
                sc = e.shape_call
                got = _status(dcopy, dcopy.trans_shape, CLASS[e.transfer_class],
                              _fmt(sc["src_format"]), sc["src_shape"], _dt(sc["dtype"]),
                              _fmt(sc["dst_format"]), 16)
            elif e.call in ("TransFormat", "TransDataFormat") and e.status != 0:
                # A failure is decided before any data moves: a fake non-NULL
                # source stands for the test's host array (NULL stays NULL).
                data = 0 if a.data_var not in case.arrays else 0x1000
                kw = dict(src_c0=a.c0[0], dst_c0=a.c0[1])
                if e.call == "TransDataFormat":
                    got = _status(dcopy, dcopy.trans_data_format, 0, data, _fmt(a.src_format),
                                  _fmt(a.dst_format), a.src_shape, a.dst_shape, _dt(a.dtype),
                                  0, **kw)
                else:
                    cls = CLASS.get(e.transfer_class, 3)
                    got = _status(dcopy, dcopy.trans_format, cls, 0, data, _fmt(a.src_format),
                                  _fmt(a.dst_format), a.src_shape, a.dst_shape, _dt(a.dtype), 0,
                                  **kw)
            else:
                continue
            assert got == e.status, (case.name, e)
            checked += 1
    assert checked >= {"nz": 15, "zz": 23, "transpose": 8}[which]


def test_trans_shape_results(dcopy):
    f = dcopy.FORMAT
    assert dcopy.trans_shape(3, f["NCHW"], [1, 3, 8, 8], 1, f["HWCN"]) == [8, 8, 3, 1]
    assert dcopy.trans_shape(3, f["NHWC"], [1, 8, 8, 3], 1, f["NCHW"]) == [1, 3, 8, 8]
    assert dcopy.trans_shape(1, f["ND"], [2, 2, 17, 4], 1, f["FRACTAL_NZ"], 16) == \
        [2, 2, 1, 2, 16, 16]
    assert dcopy.trans_tensor_shape(f["NHWC"], [2, 2, 4, 17], 0, f["FRACTAL_NZ"], 16) == \
        [2, 2, 2, 1, 16, 16]
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.trans_tensor_shape(f["FRACTAL_NZ"], [1, 1, 16, 16], 1, f["ND"], 16)
    assert e.value.code == dcopy.ERR_FORMAT_INVALID
    with pytest.raises(dcopy.DcopyError) as e:  # not a registered pair
        dcopy.trans_tensor_shape(f["ND"], [4, 4], 1, f["NC1HWC0"], 16)
    assert e.value.code == dcopy.ERR_FORMAT_INVALID
    # ND -> FRACTAL_Z is the TBE transfer: a 2-D [C, N] weight.
    assert dcopy.trans_tensor_shape(f["ND"], [17, 4], 1, f["FRACTAL_Z"], 16) == [2, 1, 16, 16]


def test_data_type_sizes(dcopy):
    d = dcopy.DATA_TYPE
    assert [dcopy.data_type_size(d[k]) for k in ("FLOAT", "FLOAT16", "INT8", "INT64", "BF16",
                                                 "COMPLEX128")] == [4, 2, 1, 8, 2, 16]
    assert dcopy.data_type_size(d["STRING"]) < 0 and dcopy.data_type_size(d["UNDEFINED"]) < 0


def test_registry_and_null_data(dcopy):
    f, d = dcopy.FORMAT, dcopy.DATA_TYPE
    # Unregistered pair -> FORMAT_INVALID before anything else (formats.cc:31-38).
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.trans_data_format(0, 0, f["ND"], f["NC1HWC0"], [4, 4], [4, 4], d["FLOAT"], 0)
    assert e.value.code == dcopy.ERR_FORMAT_INVALID
    # NULL data with a non-empty shape -> PARAM_INVALID (formats.cc:40-49).
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.trans_data_format(0, 0, f["ND"], f["FRACTAL_NZ"], [4, 4], [1, 1, 16, 16],
                                d["FLOAT16"], 0)
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    # Empty tensors succeed with length 0 and move nothing.
    assert dcopy.trans_data_format(0, 0x1000, f["ND"], f["FRACTAL_NZ"], [0, 16], [1, 0, 16, 16],
                                   d["FLOAT16"], 0) == 0
    # A result larger than the destination is refused before any launch.
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.trans_data_format(0, 0x1000, f["ND"], f["FRACTAL_NZ"], [4, 4], [1, 1, 16, 16],
                                d["FLOAT16"], 100)
    assert e.value.code == dcopy.ERR_PARAM_INVALID


def test_transpose_argument_checks(dcopy):
    d = dcopy.DATA_TYPE
    for shape, perm in [([2, 4], [0, 0]), ([2, 4], [0, 2]), ([2, -4], [1, 0]), ([], [])]:
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.transpose(0, 0x1000, shape, perm, d["UINT8"])
        assert e.value.code == dcopy.ERR_PARAM_INVALID
    with pytest.raises(dcopy.DcopyError) as e:  # NULL source (transpose.cc:80-83)
        dcopy.transpose(0, 0, [2, 2], [1, 0], d["UINT8"])
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    with pytest.raises(dcopy.DcopyError) as e:  # unsized data type
        dcopy.transpose(0, 0x1000, [2, 2], [1, 0], d["STRING"])
    assert e.value.code == dcopy.ERR_PARAM_INVALID


FZ_FILES = sorted(ge_goldens.FZ_TESTS)


def _full(dcopy, name, sub):
    """The test's full GE format: primary plus the sub format it was built with."""
    return dcopy.format_with_sub(ge_goldens.FMT[name], sub)


@pytest.mark.parametrize("which", FZ_FILES)
def test_fractal_z_expectations(dcopy, reference_root, which):
    """Every expectation of GE's FRACTAL_Z unit tests, through the C ABI without data
    movement: failures by status, TransShape by its result, and data-moving
    successes by the result length the transfer reports."""
    checked = 0
    for case in ge_goldens.load(reference_root, which):
        for e in case.expects:
            a = case.args.get(e.args) if e.args else None
            if a is None:
                continue
            src_f = _full(dcopy, a.src_format, a.src_format_sub)
            dst_f = _full(dcopy, a.dst_format, a.dst_format_sub)
            if e.call == "TransShape":
                try:
                    got_shape = dcopy.trans_shape(CLASS[e.transfer_class], src_f, a.src_shape,
                                                  ge_goldens.DT[a.dtype], dst_f, a.c0[1])
                    got = 0
                except dcopy.DcopyError as err:
                    got = dcopy.status_to_ge(err.code)
                assert got == e.status, (case.name, e)
                if got == 0:
                    assert got_shape == a.dst_shape, case.name
            else:
                cls = 0 if e.call == "TransDataFormat" else CLASS[e.transfer_class]
                data = 0 if a.data_var not in case.arrays else 0x1000
                try:
                    n = dcopy.trans_format_check(cls, data, src_f, dst_f, a.src_shape,
                                                 a.dst_shape, ge_goldens.DT[a.dtype],
                                                 src_c0=a.c0[0], dst_c0=a.c0[1],
                                                 src_sub=a.src_sub, dst_sub=a.dst_sub)
                    got = 0
                except dcopy.DcopyError as err:
                    got = dcopy.status_to_ge(err.code)
                assert got == e.status, (case.name, e, got)
                out = case.outputs.get(e.args)
                if got == 0 and out is not None:
                    assert n == case.arrays[out].nbytes, (case.name, n)
            checked += 1
    assert checked == {"hwcn_fz": 8, "nchw_fz": 10, "nhwc_fz": 10, "nd_fz": 6, "fz_nchw": 20,
                       "fz_hwcn": 17, "fz_nhwc": 14}[which]
