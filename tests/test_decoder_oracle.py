"""The DPT decoder operations of the oracle (oracle.conv3x3, conv1x1,
conv_transpose, resize_bilinear) pinned against the reference's own cases
(crates/beatlm-bench/src/reference.rs:651-720). CPU only."""
import numpy as np

import oracle


def test_a_one_hot_kernel_copies_the_input_through_the_centre_tap():
    h, w, c = 3, 4, 2
    k = np.zeros(9 * c * c, np.float32)
    for ci in range(c):
        k[(4 * c + ci) * c + ci] = 1.0
    x = np.arange(h * w * c, dtype=np.float32)
    assert np.array_equal(oracle.conv3x3(x, k, None, h, w, c, c), x)


def test_a_corner_pixel_sums_only_the_taps_inside_the_image():
    ones = np.ones(4, np.float32)
    assert list(oracle.conv3x3(ones, np.ones(9, np.float32), None, 2, 2, 1, 1)) == [4.0] * 4
    assert list(oracle.conv3x3(ones, np.ones(9, np.float32), np.array([0.5], np.float32),
                               2, 2, 1, 1)) == [4.5] * 4


def test_a_strided_convolution_samples_every_stride_th_pixel():
    h, w = 5, 4
    k = np.zeros(9, np.float32)
    k[4] = 1.0
    x = np.arange(h * w, dtype=np.float32)
    assert list(oracle.conv3x3(x, k, None, h, w, 1, 1, stride=2)) == [0, 2, 8, 10, 16, 18]
    ones = oracle.conv3x3(np.ones(20, np.float32), np.ones(9, np.float32),
                          np.array([0.5], np.float32), h, w, 1, 1, stride=2)
    assert list(ones[:2]) == [4.5, 6.5]


def test_a_1x1_convolution_is_the_matrix_product_of_its_pixels():
    x = np.arange(15, dtype=np.float32) * np.float32(0.25) - np.float32(1.0)
    w = np.float32(0.5) - np.arange(6, dtype=np.float32) * np.float32(0.3)
    b = np.array([0.1, -0.2], np.float32)
    assert np.array_equal(oracle.conv1x1(x, w, b, 5, 3, 2), oracle.matmul(x, w, b, 5, 3, 2))


def test_a_transposed_convolution_writes_one_block_per_input_pixel():
    out = oracle.conv_transpose(np.array([10.0, -1.0], np.float32),
                                np.array([1, 2, 3, 4], np.float32),
                                np.array([0.5], np.float32), 1, 2, 1, 1, 2)
    assert list(out) == [10.5, 20.5, -0.5, -1.5, 30.5, 40.5, -2.5, -3.5]


def test_aligned_corner_resampling_keeps_the_corners_and_interpolates_linearly():
    out = oracle.resize_bilinear(np.array([0, 2, 4, 6], np.float32), 2, 2, 3, 3, 1)
    assert list(out) == [0, 1, 2, 2, 3, 4, 4, 5, 6]
    wide = oracle.resize_bilinear(np.arange(4, dtype=np.float32), 1, 4, 1, 7, 1)
    assert list(wide) == [0, 0.5, 1, 1.5, 2, 2.5, 3]
    assert list(oracle.resize_bilinear(np.array([1, 9], np.float32), 2, 1, 1, 1, 1)) == [1.0]
