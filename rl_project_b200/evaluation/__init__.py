"""Evaluation: structured results, quality / reward / performance suites, benchmarks,
model inspection and regression rules."""

from rl_project_b200.core.protocols import EvaluationResult
from rl_project_b200.evaluation.performance import PerformanceSuite, measure_engine, measure_generation
from rl_project_b200.evaluation.quality import AgentAccuracySuite, HeldOutLossSuite, VerifierPassRateSuite
from rl_project_b200.evaluation.regression import RegressionReport, RegressionRule, evaluate_regression
from rl_project_b200.evaluation.results import load_results, merge_metrics, save_results
from rl_project_b200.evaluation.reward import (PreferenceWinRateSuite, RecordRewardSuite, TrajectoryRewardSuite,
                                               reward_statistics)
from rl_project_b200.evaluation.suites import BENCHMARKS, BenchmarkSuite, build_benchmark

__all__ = ["EvaluationResult", "PerformanceSuite", "measure_generation", "measure_engine", "AgentAccuracySuite",
           "HeldOutLossSuite", "VerifierPassRateSuite", "RegressionReport", "RegressionRule", "evaluate_regression",
           "load_results", "merge_metrics", "save_results", "PreferenceWinRateSuite", "RecordRewardSuite",
           "TrajectoryRewardSuite", "reward_statistics", "BENCHMARKS", "BenchmarkSuite", "build_benchmark"]
