"""Step messages with the field names of protos/distributed_inference.proto:49-79.

``WorkerExecutionEngine.execute_step`` reads requests by attribute, so it accepts
the reference's generated ``pb2.StepRequest`` as well as these dataclasses, and
returns a ``StepResponse`` dataclass that ``to_proto(pb2)`` converts back into the
reference's protobuf message for the gRPC worker service.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List


@dataclass
class SequenceSlot:
    """SequenceSlotProto (distributed_inference.proto:49-57)."""
    seq_id: str
    is_prefill: bool
    prompt_token_ids: List[int] = field(default_factory=list)
    current_token_id: int = 0
    current_len: int = 0
    block_table: List[int] = field(default_factory=list)
    slot_offset: int = 0


@dataclass
class StepRequest:
    """StepRequest (distributed_inference.proto:59-62)."""
    step_id: int
    active_sequences: List[SequenceSlot] = field(default_factory=list)


@dataclass
class SampledToken:
    """SampledTokenProto (distributed_inference.proto:64-68)."""
    seq_id: str
    token_id: int
    top_logits: List[float] = field(default_factory=list)


@dataclass
class StepResponse:
    """StepResponse (distributed_inference.proto:70-79)."""
    step_id: int
    rank: int
    success: bool
    error_message: str = ""
    sampled_tokens: List[SampledToken] = field(default_factory=list)
    step_latency_ms: float = 0.0
    active_blocks: int = 0
    free_blocks: int = 0

    def to_proto(self, pb2):
        """The equivalent ``pb2.StepResponse`` of the reference's generated module."""
        return pb2.StepResponse(
            step_id=self.step_id, rank=self.rank, success=self.success, error_message=self.error_message,
            sampled_tokens=[pb2.SampledTokenProto(seq_id=t.seq_id, token_id=t.token_id, top_logits=t.top_logits)
                            for t in self.sampled_tokens],
            step_latency_ms=self.step_latency_ms, active_blocks=self.active_blocks, free_blocks=self.free_blocks)
