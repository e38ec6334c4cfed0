"""opendm_b200: a B200-native (sm_100a) MuonAdamW optimizer step.

Drop-in for ``opendm.optimizer`` of dexmal/opendm:

    from opendm_b200.optimizer import MuonAdamW, mark_muon_parameters
"""

__version__ = "0.1.0"
