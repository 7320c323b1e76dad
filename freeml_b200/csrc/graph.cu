// Recorded launch plans: the operator entry points issued on a capture stream
// become one CUDA graph that a host runtime replays every step instead of
// dispatching each operator again (for FreeML's Model::Run over MatrixCUDA,
// whose per-operator host work -- string-keyed blob lookups, views, one C-ABI
// call each, ModelLibrary/Model.h:764-788 -- dominates small models).
#include "fml_common.cuh"

struct fml_graph
{
    cudaGraphExec_t exec = nullptr;
    uint64_t kernels = 0;  // kernels one replay launches
};

namespace fml {
namespace {
// launch-counter value at fml_capture_begin (recorded kernels do not run)
uint64_t g_capture_start = 0;
bool g_capturing = false;
}  // namespace
}  // namespace fml

using namespace fml;

extern "C" {

int fml_capture_begin(fml_stream_t* stream_out)
{
    FML_REQUIRE(stream_out, "fml_capture_begin: null argument");
    FML_REQUIRE(!g_capturing, "fml_capture_begin: a capture is already open");
    cudaStream_t s = nullptr;
    FML_CUDA_TRY(cudaStreamCreate(&s));
    const cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed);
    if (e != cudaSuccess)
    {
        cudaStreamDestroy(s);
        return set_error(FML_ERR_CUDA, "cudaStreamBeginCapture: %s", cudaGetErrorString(e));
    }
    g_capture_start = launch_counter().load();
    g_capturing = true;
    *stream_out = s;
    return FML_OK;
}

int fml_capture_end(fml_stream_t stream, fml_graph** graph_out)
{
    FML_REQUIRE(stream && graph_out, "fml_capture_end: null argument");
    FML_REQUIRE(g_capturing, "fml_capture_end: no capture is open");
    g_capturing = false;
    cudaStream_t s = as_stream(stream);
    const uint64_t recorded = launch_counter().load() - g_capture_start;
    launch_counter().fetch_sub(recorded, std::memory_order_relaxed);
    *graph_out = nullptr;
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(s, &g);
    cudaStreamDestroy(s);
    if (e != cudaSuccess) return set_error(FML_ERR_CUDA, "cudaStreamEndCapture: %s", cudaGetErrorString(e));
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return set_error(FML_ERR_CUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(e));
    auto* out = new fml_graph();
    out->exec = exec;
    out->kernels = recorded;
    *graph_out = out;
    return FML_OK;
}

int fml_graph_launch(fml_graph* graph, fml_stream_t stream)
{
    FML_REQUIRE(graph && graph->exec, "fml_graph_launch: null graph");
    FML_CUDA_TRY(cudaGraphLaunch(graph->exec, as_stream(stream)));
    launch_counter().fetch_add(graph->kernels, std::memory_order_relaxed);
    return FML_OK;
}

int fml_graph_destroy(fml_graph* graph)
{
    if (!graph) return FML_OK;
    if (graph->exec) cudaGraphExecDestroy(graph->exec);
    delete graph;
    return FML_OK;
}

}  // extern "C"
