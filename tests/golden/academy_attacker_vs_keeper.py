# A GRF scenario file (the format of GRF's gfootball/scenarios/*.py) written for this repository:
# the single-skill drill of the benchmark's second configuration. One controlled attacker starts
# with the ball a quarter of the pitch length (0.5 of GRF's 2.0-unit length) from the opponent
# goal and faces a lone built-in-AI goalkeeper in that goal. The episode ends on a goal, a change
# of possession or the ball out of play, or after 400 steps. Its bundle is built by make_drill.py.
# ruff: noqa: F403, F405

from . import *


def build_scenario(builder):
    builder.config().game_duration = 400
    builder.config().deterministic = False
    builder.config().offsides = False
    builder.config().end_episode_on_score = True
    builder.config().end_episode_on_out_of_play = True
    builder.config().end_episode_on_possession_change = True
    builder.SetBallPosition(0.52, 0.0)

    builder.SetTeam(Team.e_Left)
    builder.AddPlayer(-1.0, 0.0, e_PlayerRole_GK)
    builder.AddPlayer(0.5, 0.0, e_PlayerRole_CF)

    builder.SetTeam(Team.e_Right)
    builder.AddPlayer(-1.0, 0.0, e_PlayerRole_GK)
