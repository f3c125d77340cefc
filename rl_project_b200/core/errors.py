"""Typed framework errors.

Every error class carries a ``hint`` that tells the caller what to do next.
The class names and their inheritance match the reference's error taxonomy
(``src/forgeline/core/errors.py:11-149``) so user code that catches, say,
``CheckpointCorruptError`` keeps working; the hint texts are this project's own.
"""

from __future__ import annotations


class ForgelineError(Exception):
    """Root of every error this framework raises on purpose."""

    hint: str = ""

    def __init__(self, message: str, *, hint: str | None = None):
        super().__init__(message)
        self.message = message
        if hint is not None:
            self.hint = hint

    def __str__(self) -> str:
        if not self.hint:
            return self.message
        return f"{self.message} [hint: {self.hint}]"


FrameworkError = ForgelineError


def _family(name: str, base: type, hint: str, doc: str = "") -> type:
    cls = type(name, (base,), {"hint": hint, "__doc__": doc or hint, "__module__": __name__})
    return cls


# configuration ---------------------------------------------------------------
ConfigError = _family("ConfigError", ForgelineError,
                      "Fix the manifest field named in the message and re-run validation.")
UnknownPresetError = _family("UnknownPresetError", ConfigError,
                             "Run the `presets` CLI command to see every preset name.")

# data ------------------------------------------------------------------------
DatasetError = _family("DatasetError", ForgelineError,
                       "Check that the dataset path exists and matches the declared kind.")
MalformedRecordError = _family("MalformedRecordError", DatasetError,
                               "Repair or drop the record at the file:line given in the message.")
TokenizerError = _family("TokenizerError", ForgelineError,
                         "Provide tokenizer metadata (meta.pkl) or a resolvable tokenizer name.")

# models ----------------------------------------------------------------------
ModelError = _family("ModelError", ForgelineError,
                     "Compare the model spec with the checkpoint that is being loaded.")
IncompatibleStateError = _family("IncompatibleStateError", ModelError,
                                 "The weights come from another architecture; build the model from the checkpoint's spec.")
QuantizationError = _family("QuantizationError", ForgelineError,
                            "Check the tensor shape against the quantisation block size and format.")
ExportError = _family("ExportError", ForgelineError,
                      "Check the export format name and that the destination is writable.")

# rewards / rollouts ----------------------------------------------------------
RewardError = _family("RewardError", ForgelineError,
                      "A reward provider produced a non-finite or malformed score.")
InvalidRewardError = _family("InvalidRewardError", RewardError, RewardError.hint)
VerifierError = _family("VerifierError", ForgelineError,
                        "The verifier raised; the completion is scored as a failure.")
ToolExecutionError = _family("ToolExecutionError", ForgelineError,
                             "The tool failed or timed out; its error text becomes the observation.")
RolloutError = _family("RolloutError", ForgelineError,
                       "Generation failed; check prompt lengths against the context size.")

# checkpoints -----------------------------------------------------------------
CheckpointError = _family("CheckpointError", ForgelineError,
                          "Look at the checkpoint directory and its manifest.json.")
CheckpointNotFoundError = _family("CheckpointNotFoundError", CheckpointError,
                                  "Nothing was saved at that path yet; train first or point --resume elsewhere.")
CheckpointCorruptError = _family("CheckpointCorruptError", CheckpointError,
                                 "The directory is partial or unreadable; fall back to an older checkpoint.")
CheckpointMismatchError = _family("CheckpointMismatchError", CheckpointError,
                                  "The checkpoint belongs to another model spec or algorithm.")

# distributed -----------------------------------------------------------------
DistributedConfigError = _family("DistributedConfigError", ForgelineError,
                                 "Check WORLD_SIZE, the parallel degrees and the launcher environment.")
DistributedTimeoutError = _family("DistributedTimeoutError", DistributedConfigError,
                                  "A peer did not answer within the timeout; a rank probably died or stalled.")
KernelError = _family("KernelError", ForgelineError,
                      "A native kernel reported an error status; the message names the kernel and code.")

# evaluation / deployment -----------------------------------------------------
EvaluationError = _family("EvaluationError", ForgelineError,
                          "An evaluation suite failed; the message names the suite.")
PromotionError = _family("PromotionError", ForgelineError,
                         "A promotion gate failed closed; read the gate report.")
RegistryError = _family("RegistryError", ForgelineError,
                        "The candidate registry has no such candidate or is inconsistent.")
ServingError = _family("ServingError", ForgelineError,
                       "The serving backend failed; check the request body and model.")
BackendUnavailableError = _family("BackendUnavailableError", ServingError,
                                  "The backend is not loaded or a feature flag disabled it.")
OptionalDependencyError = _family("OptionalDependencyError", ForgelineError,
                                  "Install the optional package named in the message.")

# orchestration ---------------------------------------------------------------
OrchestrationError = _family("OrchestrationError", ForgelineError,
                             "A worker pool gave up after its retries; check worker resources and logs.")

__all__ = [n for n, v in dict(globals()).items() if isinstance(v, type) and issubclass(v, ForgelineError)]
