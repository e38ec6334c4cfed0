from .muon_adamw import (MuonAdamW, MuonShardPlan, is_default_muon_parameter, mark_muon_parameters,
                         zeropower_via_newtonschulz5)

__all__ = ["MuonAdamW", "mark_muon_parameters", "MuonShardPlan", "is_default_muon_parameter",
           "zeropower_via_newtonschulz5"]
