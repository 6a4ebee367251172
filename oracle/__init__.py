"""CPU oracle of the Polar Express step -- test infrastructure only.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU baseline
arm; never by the muon_fusion_ascend950_b200 package."""
