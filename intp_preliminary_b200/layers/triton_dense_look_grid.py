"""Drop-in for the reference's ``layers/triton_dense_look_grid.py``.

Same public name and signature (``dense_look_grid_sample``, :184-202); the
implementation is the sm_100a kernel library, not Triton.  The reference's
explicit sampler ``reference_dense_look_grid_sample`` is test infrastructure
and lives in the repository's ``oracle`` package.
"""

from ..dense_look_grid import dense_look_grid_sample

__all__ = ["dense_look_grid_sample"]
