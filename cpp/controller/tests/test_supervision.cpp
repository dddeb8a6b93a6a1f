// Supervisor contracts with the test binary itself as the fake worker (--child mode).
#include <signal.h>
#include <unistd.h>

#include <chrono>
#include <iostream>
#include <string>
#include <thread>

#include "check.hpp"
#include "ds/process.hpp"

using namespace ds;

static std::string self_path;

// fake worker: echoes ops; special ops exercise the supervisor
static int child_main() {
  std::string line;
  while (std::getline(std::cin, line)) {
    Json req = Json::parse(line);
    const std::string op = req.at("op").as_string();
    Json reply = Json::object();
    reply["version"] = 1;
    reply["id"] = req.at("id");
    if (op == "sleep") {
      std::this_thread::sleep_for(std::chrono::milliseconds(req.integer("ms", 0)));
    } else if (op == "wrong_id") {
      reply["id"] = 999999;
    } else if (op == "big") {
      Json r = Json::object();
      r["blob"] = std::string(static_cast<size_t>(req.integer("bytes", 0)), 'x');
      reply["ok"] = true;
      reply["result"] = r;
      std::cout << reply.dump() << "\n" << std::flush;
      continue;
    } else if (op == "split") {
      reply["ok"] = true;
      reply["result"] = Json::object();
      const std::string text = reply.dump();
      std::cout << text.substr(0, 5) << std::flush;
      std::this_thread::sleep_for(std::chrono::milliseconds(50));
      std::cout << text.substr(5) << "\n" << std::flush;
      continue;
    } else if (op == "fail") {
      reply["ok"] = false;
      reply["error"] = "requested failure";
      std::cout << reply.dump() << "\n" << std::flush;
      continue;
    } else if (op == "grandchild") {
      if (fork() == 0) {  // stays in our process group
        execl("/bin/sleep", "sleep", "30", nullptr);
        _exit(127);
      }
    } else if (op == "exit") {
      _exit(3);
    } else if (op == "ignore_term") {
      signal(SIGTERM, SIG_IGN);
    }
    reply["ok"] = true;
    reply["result"] = req;
    std::cout << reply.dump() << "\n" << std::flush;
  }
  return 0;
}

static WorkerProcess spawn() { return WorkerProcess({self_path, "--child"}, {{"DS_FAKE", "1"}}, "/dev/null"); }

TEST("envelope round trip with versioned ids") {
  auto w = spawn();
  Json r = w.call("echo", Json::parse(R"({"x":[1,2,3]})"), 10);
  CHECK(r.at("x")[2].as_int() == 3 && r.at("op").as_string() == "echo" && r.at("version").as_int() == 1);
  CHECK(w.stop());
}

TEST("split and large replies are reassembled") {
  auto w = spawn();
  CHECK(w.call("split", Json::object(), 10).is_object());
  Json big = Json::object();
  big["bytes"] = 3 << 20;
  CHECK(w.call("big", big, 30).at("blob").size() == static_cast<size_t>(3 << 20));
  CHECK(w.stop());
}

TEST("deadline expiry raises WorkerDeadlineExceeded") {
  auto w = spawn();
  Json s = Json::object();
  s["ms"] = 2000;
  bool threw = false;
  try {
    w.call("sleep", s, 0.2);
  } catch (const WorkerDeadlineExceeded&) {
    threw = true;
  }
  CHECK(threw);
  CHECK(w.stop(0.5));
}

TEST("heartbeat can cancel a call") {
  auto w = spawn();
  Json s = Json::object();
  s["ms"] = 3000;
  int beats = 0;
  bool threw = false;
  try {
    w.call("sleep", s, 10, [&](CancelScope& c) {
      if (++beats >= 2) c.cancel("test");
    });
  } catch (const WorkerDeadlineExceeded& e) {
    threw = std::string(e.what()).find("cancelled") != std::string::npos;
  }
  CHECK(threw && beats == 2);
  CHECK(w.stop(0.5));
}

TEST("wrong reply id and ok=false are reported") {
  auto w = spawn();
  CHECK_THROWS(w.call("fail", Json::object(), 5));
  bool proto = false;
  try {
    w.call("wrong_id", Json::object(), 5);
  } catch (const WorkerProtocolError&) {
    proto = true;
  }
  CHECK(proto);
  CHECK(w.stop());
}

TEST("a dead worker surfaces as WorkerFailure") {
  auto w = spawn();
  bool failed = false;
  try {
    w.call("exit", Json::object(), 5);
  } catch (const WorkerFailure&) {
    failed = true;
  }
  CHECK(failed);
  // the reply pipe closes just before the process is reaped: allow the exit to land
  for (int i = 0; i < 500 && w.alive(); ++i) std::this_thread::sleep_for(std::chrono::milliseconds(10));
  CHECK(!w.alive());
  CHECK(w.stop());
}

TEST("stop reaps grandchildren and escalates past ignored SIGTERM") {
  auto w = spawn();
  w.call("grandchild", Json::object(), 5);
  w.call("ignore_term", Json::object(), 5);
  const pid_t pg = w.pid();
  CHECK(kill(-pg, 0) == 0);
  CHECK(w.stop(0.3));
  CHECK(kill(-pg, 0) != 0);
}

int main(int argc, char** argv) {
  self_path = argv[0];
  if (argc > 1 && std::string(argv[1]) == "--child") return child_main();
  become_subreaper();
  return dstest::run_all();
}
