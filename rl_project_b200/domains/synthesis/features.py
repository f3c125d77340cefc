"""128-d state vectors of synthesis records: 8 normalised condition / outcome
features, a 100-bit molecule fingerprint, zero padding."""

from __future__ import annotations

import hashlib
from typing import Dict, List

import torch

from rl_project_b200.domains.synthesis.reward import extract_outcomes

STATE_DIM = 128
FP_BITS = 100

MOLECULE_SMILES = {
    "Aspirin": "CC(=O)OC1=CC=CC=C1C(=O)O",
    "Ibuprofen": "CC(C)CC1=CC=C(C=C1)C(C)C(=O)O",
    "Naproxen": "COC1=CC2=C(C=C1)C=C(C=C2)C(C)C(=O)O",
    "Paracetamol": "CC(=O)NC1=CC=C(C=C1)O",
    "Ketoprofen": "CC(C1=CC(=CC=C1)C(=O)C2=CC=CC=C2)C(=O)O",
}

_CACHE: Dict[str, List[float]] = {}


def _hashed_fingerprint(smiles: str, n_bits: int) -> List[float]:
    """Substructure-free stand-in: each SMILES character 1..4-gram sets one hashed bit."""
    bits = [0.0] * n_bits
    for n in range(1, 5):
        for i in range(len(smiles) - n + 1):
            h = int.from_bytes(hashlib.blake2b(smiles[i:i + n].encode(), digest_size=4).digest(), "little")
            bits[h % n_bits] = 1.0
    return bits


def molecule_fingerprint(name: str, n_bits: int = FP_BITS) -> List[float]:
    """Morgan fingerprint (radius 2) through RDKit when installed, else a hashed SMILES n-gram
    fingerprint; zeros for unknown molecules."""
    key = f"{name}:{n_bits}"
    if key in _CACHE:
        return _CACHE[key]
    smiles = MOLECULE_SMILES.get(name)
    bits = [0.0] * n_bits
    if smiles:
        try:
            from rdkit import Chem
            from rdkit.Chem import AllChem

            mol = Chem.MolFromSmiles(smiles)
            fp = AllChem.GetMorganFingerprintAsBitVect(mol, radius=2, nBits=n_bits)
            bits = [float(c == "1") for c in fp.ToBitString()]
        except Exception:  # noqa: BLE001 - RDKit missing or failed
            bits = _hashed_fingerprint(smiles, n_bits)
    _CACHE[key] = bits
    return bits


def encode_trajectory(record: Dict) -> torch.Tensor:
    o = extract_outcomes(record)
    state = torch.zeros(STATE_DIM)
    state[:8] = torch.tensor([o["temperature"] / 200.0, o["time"] / 12.0, min(o["catalyst"], 1.0), o["solvent"] / 6.0,
                              o["yield"], o["selectivity"], 1.0 - o["safety_risk"], o["steps"] / 10.0])
    state[8:8 + FP_BITS] = torch.tensor(molecule_fingerprint(record.get("molecule", "")))
    return state
