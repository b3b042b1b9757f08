"""Error convention of the inference path.

Every rejected input, unsupported configuration or failed device call is raised
as ``ContractError`` (a ``ValueError``), matching reference
``src/nnunet_mlx/errors.py:4``; the C-ABI's nonzero status codes are mapped to
it by ``nnunet_mlx_b200._native``.
"""


class ContractError(ValueError):
    """A request, model or device result violates the inference contract."""
