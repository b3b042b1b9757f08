"""Device preprocessing against the reference's own ``preprocess_raw_case`` outputs (needs a B200).

The outputs were recorded by ``tests/golden/make_golden.py`` from the reference's
``data/preprocessing.py:60-163`` on grid-preserving plans (nine cases: every normalisation scheme,
masks with holes, transposes, input dtypes, a cascade input).  Bars as in
``test_gpu_preprocess.py``: bitwise, except within rtol 1e-5 / atol 5e-6 where a z-score mean and
standard deviation are reduced.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from .conftest import GOLDEN
from .test_gpu_preprocess import ATOL, RTOL, _status_clean

pytestmark = pytest.mark.gpu


def test_device_preprocessing_matches_reference_outputs(cuda_device):
    """The device path against the reference's own ``preprocess_raw_case`` outputs (recorded).

    Nine grid-preserving cases: every normalisation scheme, masks with holes, transposes, input
    dtypes, a cascade input.  Bitwise except where a z-score mean and standard deviation are reduced.
    """
    from nnunet_mlx_b200.data.preprocessing import PreprocessingPlans, preprocess_raw_case

    saved = np.load(GOLDEN / "preprocess_reference.npz")
    for case in json.loads(str(saved["metadata"].item()))["cases"]:
        name = case["name"]
        plans = PreprocessingPlans.from_payload(case["plans"], configuration="selected")
        previous = saved[f"{name}-previous"] if f"{name}-previous" in saved.files else None
        result = preprocess_raw_case(saved[f"{name}-raw"], {"spacing": case["spacing"]}, plans,
                                     segmentation_previous_stage=previous, device=cuda_device)
        assert result.properties["bbox_used_for_cropping"] == case["bbox"], name
        got, expected = result.data.cpu().numpy(), saved[f"{name}-data"]
        if "ZScoreNormalization" in plans.normalization_schemes:
            np.testing.assert_allclose(got, expected, rtol=RTOL, atol=ATOL, err_msg=name)
        else:
            np.testing.assert_array_equal(got, expected, err_msg=name)
        if previous is not None:
            np.testing.assert_array_equal(result.previous_stage.cpu().numpy(),
                                          saved[f"{name}-labels"].astype(np.int64), err_msg=name)
    _status_clean()
