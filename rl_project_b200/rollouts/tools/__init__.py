"""Tool execution and tagged-output parsing for agent rollouts."""

from rl_project_b200.rollouts.tools.parser import ParsedOutput, ToolCall, format_tool_result, parse_tagged_output
from rl_project_b200.rollouts.tools.python_executor import ExecutionResult, PythonExecutorTool, execute_python
