"""lnet_b200: B200-native (sm_100a) ALPHABET forward path and pole-residue
Laplace layer behind the reference ``lnet`` module API.

* :class:`B200Alphabet` — drop-in for ``lnet.Alphabet`` (same state_dict,
  same forward signature and metadata errors).
* :class:`B200PoleResidueTemporalMixing` — drop-in for
  ``lnet.laplace.PoleResidueTemporalMixing``.
* :mod:`lnet_b200.ops` — the same calls as ``torch.library`` custom ops with
  ``register_fake`` meta kernels (``lnet_b200::alphabet_forward``,
  ``lnet_b200::laplace_forward``, ``lnet_b200::patchify_images``).
* :mod:`lnet_b200.inference` — ``prepare_compiled_inference`` /
  ``prepare_maskless_inference`` with the reference's call surface.
* :mod:`lnet_b200.sharding` — batch sharding over one process per GPU.
* :mod:`lnet_b200.channelsplit` — mode (channel) split over ranks (one
  all-reduce of the writer stream, one all-gather of moment sums).
* :mod:`lnet_b200.timesplit` — sequence split over ranks (one carry exchange
  per block) for requests with fewer rows than GPUs.
* :mod:`lnet_b200.images` — uint8 images -> normalised 4x4 patch tokens on the
  GPU (:meth:`B200Alphabet.forward_images`).
* :mod:`lnet_b200.pipeline` — host-fed serving loop overlapping the copies of
  the next batch with the current forward.
* :mod:`lnet_b200.graph` — CUDA-graph capture and replay of a prepared forward.

All compute runs in the C-ABI CUDA library ``_lib/liblnet_b200.so`` built by
:func:`lnet_b200.build.build`; there is no CPU fallback.
"""

from . import ops  # registers the lnet_b200:: custom ops
from .alphabet import AlphabetConfig, B200Alphabet
from .inference import prepare_compiled_inference, prepare_maskless_inference
from .train_runtime import (
    AlphabetTrainingRuntime,
    prepare_aggressive_training,
    prepare_exact_split_training,
)
from .laplace import (
    B200PoleResidueTemporalMixing,
    LaplaceParameterError,
    LaplaceShapeError,
)

__all__ = [
    "AlphabetConfig",
    "AlphabetTrainingRuntime",
    "B200Alphabet",
    "B200PoleResidueTemporalMixing",
    "LaplaceParameterError",
    "LaplaceShapeError",
    "ops",
    "prepare_aggressive_training",
    "prepare_compiled_inference",
    "prepare_exact_split_training",
    "prepare_maskless_inference",
]
